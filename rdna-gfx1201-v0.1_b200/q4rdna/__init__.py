"""Python host layer of the B200 Q4_RDNA GEMV (ctypes over include/q4rdna.h).

The compute is the CUDA library ``libq4rdna.so`` next to this file; this module
only passes pointers.  PyTorch, where used, is plumbing for device buffers and
streams.  There is no CPU fallback: without the library every call raises.

The operator surface mirrors the reference's ggml hooks
(source/q4rdna.cuh:5-24): ``mul_mat``, ``mul_mat_add`` and ``mul_mat_glu`` take
a ggml tensor name plus shapes and return True when the work was enqueued,
False when the caller must fall back to its stock kernel.

The library is mapped on first use (``q4rdna.lib``, or any call), not at
import: ``import q4rdna.synth`` or ``q4rdna.format`` alone loads no CUDA code.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_int, c_int64, c_size_t, c_uint64, c_void_p

from . import format, synth  # noqa: F401

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libq4rdna.so")

OK = 0
OP_PLAIN, OP_ADD, OP_SWIGLU = 0, 1, 2
FORMAT_Q4RDNA, FORMAT_Q4K = 0, 1
Q4K_BLOCK, Q4K_BLOCK_BYTES = 256, 144
MAX_BATCH = 16
STATUS = {
    0: "OK", 1: "INVALID_ARGUMENT", 2: "SHAPE", 3: "ALIGNMENT", 4: "WORKSPACE", 5: "UNSUPPORTED",
    6: "CUDA", 7: "IO", 8: "FORMAT", 9: "NOT_FOUND", 10: "DEVICE", 11: "TOO_LARGE",
}


class Q4RDNAError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        super().__init__(f"q4rdna: {STATUS.get(status, status)} ({status_string(status)}){': ' + what if what else ''}")


CFG_OVERLAP_PREVIOUS = 1


class Cfg(ctypes.Structure):
    _fields_ = [("split", c_int), ("flags", c_int), ("reserved", c_int * 6)]


class GemvDesc(ctypes.Structure):
    _fields_ = [("tiles", c_void_p), ("gate_tiles", c_void_p), ("x", c_void_p), ("add", c_void_p),
                ("y", c_void_p), ("N", c_int), ("K", c_int), ("op", c_int), ("split", c_int),
                ("norm_weight", c_void_p), ("norm_eps", ctypes.c_float), ("format", c_int)]


class PlanInfo(ctypes.Structure):
    _fields_ = [("count", c_int), ("batch", c_int), ("items", c_int64), ("grid", c_int),
                ("weight_bytes", c_uint64), ("algo_bytes", c_uint64), ("workspace_bytes", c_size_t)]


def _bind(lib):
    P = c_void_p
    sig = {
        "q4rdna_status_string": (c_char_p, [c_int]),
        "q4rdna_version": (c_char_p, []),
        "q4rdna_select_split": (c_int, [c_int, c_int, c_int, c_int]),
        "q4rdna_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, POINTER(Cfg)]),
        "q4rdna_workspace_init": (c_int, [P, c_size_t, P]),
        "q4rdna_gemv": (c_int, [P, P, P, c_int, c_int, c_int, POINTER(Cfg), P, c_size_t, P]),
        "q4rdna_gemv_add": (c_int, [P, P, P, P, c_int, c_int, c_int, POINTER(Cfg), P, c_size_t, P]),
        "q4rdna_gemv_swiglu": (c_int, [P, P, P, P, c_int, c_int, c_int, POINTER(Cfg), P, c_size_t, P]),
        "q4rdna_dequant_f32": (c_int, [P, P, c_int, c_int, P]),
        "q4rdna_gemv_rmsnorm": (c_int, [P, P, P, P, ctypes.c_float, P, P, c_int, c_int, c_int, c_int, POINTER(Cfg), P,
                                        c_size_t, P]),
        "q4rdna_pack_bf16": (c_int, [P, P, c_int, c_int, P]),
        "q4rdna_q4k_bytes": (c_size_t, [c_int, c_int]),
        "q4rdna_q4k_gemv": (c_int, [P, P, P, P, c_int, c_int, c_int, P]),
        "q4rdna_q4k_dequant_f32": (c_int, [P, P, c_int, c_int, P]),
        "q4rdna_gemv_noalloc": (c_int, [P, P, P, c_int, c_int, c_int, POINTER(Cfg), P]),
        "q4rdna_plan_create": (c_int, [POINTER(GemvDesc), c_int, c_int, POINTER(P)]),
        "q4rdna_plan_run": (c_int, [P, P]),
        "q4rdna_plan_get_info": (c_int, [P, POINTER(PlanInfo)]),
        "q4rdna_plan_destroy": (None, [P]),
        "q4rdna_plan_run_host": (c_int, [P, P, P, c_size_t, P, P, c_size_t, c_int, P]),
        "q4rdna_plan_set_segments": (c_int, [P, c_int]),
        "q4rdna_plan_run_many": (c_int, [POINTER(P), c_int, P]),
        "q4rdna_plan_set_flags": (c_int, [P, c_int]),
        "q4rdna_plan_set_gather": (c_int, [P, c_int, c_int, P, c_size_t, POINTER(P), POINTER(P), POINTER(P)]),
        "q4rdna_plan_gather_parity": (c_int, [P]),
        "q4rdna_plan_set_gather_timeout": (c_int, [P, ctypes.c_uint32]),
        "q4rdna_ipc_alloc": (c_int, [c_size_t, POINTER(P), ctypes.c_char_p]),
        "q4rdna_ipc_open": (c_int, [ctypes.c_char_p, POINTER(P)]),
        "q4rdna_ipc_close": (c_int, [P]),
        "q4rdna_ipc_free": (c_int, [P]),
        "q4rdna_sidecar_open": (c_int, [c_char_p, c_int, POINTER(P)]),
        "q4rdna_sidecar_close": (None, [P]),
        "q4rdna_sidecar_count": (c_int, [P]),
        "q4rdna_sidecar_entry": (c_int, [P, c_int, c_char_p, POINTER(c_int), POINTER(c_int), POINTER(c_uint64)]),
        "q4rdna_sidecar_find": (c_int, [P, c_char_p, POINTER(c_int), POINTER(c_int), POINTER(P)]),
        "q4rdna_mul_mat": (c_int, [c_char_p, c_int64, c_int64, P, c_int64, P, c_int64, P]),
        "q4rdna_mul_mat_add": (c_int, [c_char_p, c_int64, c_int64, P, c_int64, P, c_int64, P, c_int64, P]),
        "q4rdna_mul_mat_glu": (c_int, [c_char_p, c_int64, c_int64, c_char_p, c_int64, c_int64, P, c_int64, P,
                                       c_int64, P]),
        "q4rdna_launch_count": (c_uint64, []),
        "q4rdna_take_fault": (ctypes.c_uint32, []),
        "q4rdna_registry_hits": (c_uint64, [c_char_p]),
        "q4rdna_report_stats": (None, []),
        "q4rdna_registry_reset": (None, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_lib_handle = None


def _load_lib():
    """The bound library, mapped on the first call; None when it was not built."""
    global _lib_handle
    if _lib_handle is None and os.path.exists(LIB_PATH):
        _lib_handle = _bind(ctypes.CDLL(LIB_PATH))
    return _lib_handle


def __getattr__(name):
    # ``q4rdna.lib``: the ctypes library (None if not built), mapped lazily
    if name == "lib":
        return _load_lib()
    raise AttributeError(f"module 'q4rdna' has no attribute {name!r}")


SYMBOLS = [
    "q4rdna_status_string", "q4rdna_version", "q4rdna_select_split", "q4rdna_workspace_bytes",
    "q4rdna_workspace_init", "q4rdna_gemv", "q4rdna_gemv_add", "q4rdna_gemv_swiglu", "q4rdna_dequant_f32", "q4rdna_pack_bf16",
    "q4rdna_gemv_rmsnorm",
    "q4rdna_gemv_noalloc",
    "q4rdna_q4k_bytes", "q4rdna_q4k_gemv", "q4rdna_q4k_dequant_f32",
    "q4rdna_plan_create", "q4rdna_plan_run", "q4rdna_plan_get_info", "q4rdna_plan_destroy",
    "q4rdna_plan_run_host", "q4rdna_plan_set_segments", "q4rdna_plan_run_many", "q4rdna_plan_set_flags", "q4rdna_plan_set_gather", "q4rdna_plan_gather_parity",
    "q4rdna_plan_set_gather_timeout", "q4rdna_ipc_alloc", "q4rdna_ipc_open",
    "q4rdna_ipc_close", "q4rdna_ipc_free",
    "q4rdna_sidecar_open", "q4rdna_sidecar_close", "q4rdna_sidecar_count", "q4rdna_sidecar_entry",
    "q4rdna_sidecar_find", "q4rdna_mul_mat", "q4rdna_mul_mat_add", "q4rdna_mul_mat_glu",
    "q4rdna_launch_count", "q4rdna_take_fault", "q4rdna_registry_hits", "q4rdna_report_stats", "q4rdna_registry_reset",
]


def _lib():
    lib = _load_lib()
    if lib is None:
        raise RuntimeError(f"q4rdna CUDA library not built: {LIB_PATH} is missing (run __graft_entry__.build())")
    return lib


def status_string(st: int) -> str:
    return _lib().q4rdna_status_string(st).decode()


def version() -> str:
    return _lib().q4rdna_version().decode()


def check(st: int, what: str = "") -> None:
    if st != OK:
        raise Q4RDNAError(st, what)


def launch_count() -> int:
    return int(_lib().q4rdna_launch_count())


def take_fault() -> int:
    """Device fault flags since the last call (0 = none); synchronises the device."""
    return int(_lib().q4rdna_take_fault())


def _cfg(split: int, flags: int = 0):
    c = Cfg()
    c.split = int(split)
    c.flags = int(flags)
    return ctypes.byref(c)


def select_split(N: int, K: int, B: int = 1, op: int = OP_PLAIN) -> int:
    return int(_lib().q4rdna_select_split(N, K, B, op))


def workspace_bytes(N: int, K: int, B: int = 1, op: int = OP_PLAIN, split: int = 0) -> int:
    return int(_lib().q4rdna_workspace_bytes(N, K, B, op, _cfg(split)))


# ------------------------------------------------------------ torch plumbing

def _stream_handle(stream=None):
    import torch

    s = torch.cuda.current_stream() if stream is None else stream
    return c_void_p(s.cuda_stream)


_WS = {}


def _workspace(nbytes: int, device, stream):
    """A zeroed device workspace of >= nbytes for this (device, stream)."""
    import torch

    if nbytes == 0:
        return None, 0
    key = (device.index if device.index is not None else torch.cuda.current_device(), stream.value)
    ws = _WS.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(nbytes + 256, dtype=torch.uint8, device=device)
        _WS[key] = ws
    return c_void_p(ws.data_ptr()), ws.numel()


def _rows(tiles, K: int) -> int:
    n = tiles.numel() * 64
    if K <= 0 or K % 64 or n % (34 * K):
        raise ValueError("tile buffer size does not match K")
    return n // (34 * K)


def gemv(tiles, x, *, op: int = OP_PLAIN, add=None, gate_tiles=None, out=None, split: int = 0, stream=None,
         norm_weight=None, norm_eps: float = 1e-6):
    """y = W x (op PLAIN), W x + add (ADD) or (W x) * silu(W_gate x) (SWIGLU).

    tiles / gate_tiles: uint8 CUDA tensors in the packed layout; x: f32 [B, K]
    or [K]; add: f32 [B, N].  Returns f32 [B, N] (or [N]).  With norm_weight
    (f32 [K]) x is the raw hidden state h and the GEMV input is
    RMSNorm(h) * norm_weight, fused (q4rdna_gemv_rmsnorm).
    """
    import torch

    squeeze = x.dim() == 1
    x2 = x.reshape(1, -1) if squeeze else x
    B, K = x2.shape
    N = _rows(tiles, K)
    if out is None:
        out = torch.empty((B, N), dtype=torch.float32, device=x.device)
    st = _stream_handle(stream)
    nbytes = workspace_bytes(N, K, B, op, split)
    ws, wsn = _workspace(nbytes, x.device, st)
    L = _lib()
    if norm_weight is not None:
        rc = L.q4rdna_gemv_rmsnorm(tiles.data_ptr(), gate_tiles.data_ptr() if gate_tiles is not None else None,
                                   x2.data_ptr(), norm_weight.data_ptr(), norm_eps,
                                   add.data_ptr() if add is not None else None, out.data_ptr(), N, K, B, op,
                                   _cfg(split), ws, wsn, st)
    elif op == OP_PLAIN:
        rc = L.q4rdna_gemv(tiles.data_ptr(), x2.data_ptr(), out.data_ptr(), N, K, B, _cfg(split), ws, wsn, st)
    elif op == OP_ADD:
        rc = L.q4rdna_gemv_add(tiles.data_ptr(), x2.data_ptr(), add.data_ptr(), out.data_ptr(), N, K, B,
                               _cfg(split), ws, wsn, st)
    elif op == OP_SWIGLU:
        rc = L.q4rdna_gemv_swiglu(tiles.data_ptr(), gate_tiles.data_ptr(), x2.data_ptr(), out.data_ptr(), N, K,
                                  B, _cfg(split), ws, wsn, st)
    else:
        raise ValueError(f"unknown op {op}")
    check(rc, f"gemv N={N} K={K} B={B}")
    return out.reshape(-1) if squeeze else out


def _q4k_rows(blocks, K: int) -> int:
    if K <= 0 or K % Q4K_BLOCK:
        raise ValueError("Q4_K needs K % 256 == 0")
    row = (K // Q4K_BLOCK) * Q4K_BLOCK_BYTES
    if blocks.numel() % row:
        raise ValueError("Q4_K buffer size does not match K")
    return blocks.numel() // row


def q4k_gemv(blocks, x, *, add=None, out=None, stream=None):
    """y = W x (+ add) for a Q4_K tensor (ggml block_q4_K rows, uint8 CUDA
    tensor); x f32 [B, K] or [K], add f32 [B, N].  Returns f32 [B, N] (or [N])."""
    import torch

    squeeze = x.dim() == 1
    x2 = x.reshape(1, -1) if squeeze else x
    B, K = x2.shape
    N = _q4k_rows(blocks, K)
    if out is None:
        out = torch.empty((B, N), dtype=torch.float32, device=x.device)
    rc = _lib().q4rdna_q4k_gemv(blocks.data_ptr(), x2.data_ptr(), add.data_ptr() if add is not None else None,
                                out.data_ptr(), N, K, B, _stream_handle(stream))
    check(rc, f"q4k_gemv N={N} K={K} B={B}")
    return out.reshape(-1) if squeeze else out


def q4k_dequant(blocks, N: int, K: int, stream=None):
    import torch

    W = torch.empty((N, K), dtype=torch.float32, device=blocks.device)
    check(_lib().q4rdna_q4k_dequant_f32(blocks.data_ptr(), W.data_ptr(), N, K, _stream_handle(stream)),
          "q4k_dequant")
    return W


def dequant(tiles, N: int, K: int, stream=None):
    import torch

    W = torch.empty((N, K), dtype=torch.float32, device=tiles.device)
    check(_lib().q4rdna_dequant_f32(tiles.data_ptr(), W.data_ptr(), N, K, _stream_handle(stream)), "dequant")
    return W


def pack_bf16(w, stream=None):
    """Q4_RDNA tiles (uint8 CUDA tensor, N*K*34/64 bytes) of a bf16 matrix
    [N, K] (torch.bfloat16, or its raw bits as int16/uint16, on the GPU), byte
    for byte what the reference packer writes (q4rdna_pack_bf16)."""
    import torch

    if w.dim() != 2 or not w.is_cuda:
        raise ValueError("pack_bf16 takes a 2-D CUDA tensor")
    if w.dtype not in (torch.bfloat16, torch.int16, torch.uint16):
        raise ValueError("pack_bf16 takes bfloat16 weights (or their 16-bit patterns)")
    w = w.contiguous()
    N, K = w.shape
    out = torch.empty(N * K * 34 // 64, dtype=torch.uint8, device=w.device)
    check(_lib().q4rdna_pack_bf16(w.data_ptr(), out.data_ptr(), N, K, _stream_handle(stream)), "pack_bf16")
    return out


def pack_sidecar(path: str, tensors, stream=None):
    """Writes a .q4rdna sidecar: tensors is a list of (ggml name, bf16 CUDA
    tensor [N, K]); every tensor is packed on the GPU and the container is laid
    out exactly as the reference packer lays it out (q4rdna.format)."""
    import torch

    packed = []
    for name, w in tensors:
        t = pack_bf16(w, stream)
        packed.append((name, t, w.shape[0], w.shape[1]))
    torch.cuda.synchronize()
    return format.write_sidecar(path, [(n, t.cpu().numpy(), r, c) for n, t, r, c in packed])


class Plan:
    """Many independent GEMVs in one persistent launch (q4rdna_plan_*).

    ``descs``: list of dicts with keys tiles, x, y (torch CUDA tensors) and
    optional op, add, gate_tiles, split, norm_weight, norm_eps (fused RMSNorm:
    x is then the raw hidden state) and format (FORMAT_Q4RDNA, the default, or
    FORMAT_Q4K: ``tiles`` then holds ggml block_q4_K rows).  The tensors must
    stay alive; x may be rewritten in place between runs.
    """

    def __init__(self, descs, B: int = 1):
        arr = (GemvDesc * len(descs))()
        self._keep = descs
        for i, d in enumerate(descs):
            K = d["x"].shape[-1]
            arr[i].tiles = d["tiles"].data_ptr()
            arr[i].gate_tiles = d["gate_tiles"].data_ptr() if d.get("gate_tiles") is not None else None
            arr[i].x = d["x"].data_ptr()
            arr[i].add = d["add"].data_ptr() if d.get("add") is not None else None
            arr[i].y = d["y"].data_ptr()
            fmt = d.get("format", FORMAT_Q4RDNA)
            arr[i].format = fmt
            arr[i].N = _q4k_rows(d["tiles"], K) if fmt == FORMAT_Q4K else _rows(d["tiles"], K)
            arr[i].K = K
            arr[i].op = d.get("op", OP_PLAIN)
            arr[i].split = d.get("split", 0)
            arr[i].norm_weight = d["norm_weight"].data_ptr() if d.get("norm_weight") is not None else None
            arr[i].norm_eps = d.get("norm_eps", 1e-6)
        h = c_void_p()
        check(_lib().q4rdna_plan_create(arr, len(descs), B, ctypes.byref(h)), "plan_create")
        self._h = h

    def run(self, stream=None):
        check(_lib().q4rdna_plan_run(self._h, _stream_handle(stream)), "plan_run")

    def set_flags(self, flags: int):
        """Launch options of the runs (q4rdna_plan_set_flags), e.g.
        CFG_OVERLAP_PREVIOUS: programmatic dependent launch (B = 1..2)."""
        check(_lib().q4rdna_plan_set_flags(self._h, flags), "plan_set_flags")

    def set_segments(self, segments: int):
        """run() as `segments` overlapping launches (q4rdna_plan_set_segments;
        1 or 0 = one launch, the default)."""
        check(_lib().q4rdna_plan_set_segments(self._h, segments), "plan_set_segments")

    def run_host(self, x_host, x_dev, y_dev, y_host, segments: int = 0, stream=None):
        """One run from host memory (q4rdna_plan_run_host): x_host -> x_dev,
        the GEMVs, y_dev -> y_host, in `segments` overlapped pieces (0: the library default).
        x_dev / y_dev must contain every descriptor's x / y; the host tensors
        (pinned) mirror them byte for byte."""
        for t in (x_host, x_dev, y_dev, y_host):
            if not t.is_contiguous():
                raise ValueError("run_host needs contiguous buffers")
        if x_host.nbytes != x_dev.nbytes or y_host.nbytes != y_dev.nbytes:
            raise ValueError("host and device buffers differ in size")
        check(_lib().q4rdna_plan_run_host(self._h, x_host.data_ptr(), x_dev.data_ptr(), x_dev.nbytes,
                                          y_dev.data_ptr(), y_host.data_ptr(), y_dev.nbytes, segments,
                                          _stream_handle(stream)), "plan_run_host")

    def info(self) -> dict:
        i = PlanInfo()
        check(_lib().q4rdna_plan_get_info(self._h, ctypes.byref(i)), "plan_info")
        return {k: getattr(i, k) for k, _ in PlanInfo._fields_}

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            _lib().q4rdna_plan_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def run_plans(plans, stream=None):
    """Runs the plans in order on the stream with one library call
    (q4rdna_plan_run_many); each as Plan.run would."""
    arr = (c_void_p * len(plans))(*[p._h.value for p in plans])
    check(_lib().q4rdna_plan_run_many(arr, len(plans), _stream_handle(stream)), "plan_run_many")


class Sidecar:
    """A loaded .q4rdna sidecar (q4rdna_sidecar_*): tiles live on `device`."""

    def __init__(self, path: str, device: int = 0):
        h = c_void_p()
        check(_lib().q4rdna_sidecar_open(path.encode(), device, ctypes.byref(h)), f"sidecar_open {path}")
        self._h = h

    def __len__(self):
        return int(_lib().q4rdna_sidecar_count(self._h))

    def entries(self):
        out = []
        for i in range(len(self)):
            name = ctypes.create_string_buffer(64)
            r, c, off = c_int(), c_int(), c_uint64()
            check(_lib().q4rdna_sidecar_entry(self._h, i, name, ctypes.byref(r), ctypes.byref(c), ctypes.byref(off)))
            out.append((name.value.decode(), r.value, c.value, off.value))
        return out

    def find(self, name: str):
        """(rows, cols, device address) or None if absent."""
        r, c, p = c_int(), c_int(), c_void_p()
        st = _lib().q4rdna_sidecar_find(self._h, name.encode(), ctypes.byref(r), ctypes.byref(c), ctypes.byref(p))
        if st == 9:
            return None
        check(st, f"sidecar_find {name}")
        return r.value, c.value, p.value

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            _lib().q4rdna_sidecar_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------- reference operator surface

def mul_mat(weight_name: str, weight_ne, x, dst, stream=None) -> bool:
    """ggml_cuda_q4rdna_mul_mat: weight_ne = (ne0 = K, ne1 = N); x f32 [K]; dst f32 [N]."""
    return bool(_lib().q4rdna_mul_mat(weight_name.encode(), weight_ne[0], weight_ne[1], x.data_ptr(), x.numel(),
                                      dst.data_ptr(), dst.numel(), _stream_handle(stream)))


def mul_mat_add(weight_name: str, weight_ne, x, add, dst, stream=None) -> bool:
    """ggml_cuda_q4rdna_mul_mat_add: dst = W x + add."""
    return bool(_lib().q4rdna_mul_mat_add(weight_name.encode(), weight_ne[0], weight_ne[1], x.data_ptr(),
                                          x.numel(), add.data_ptr(), add.numel(), dst.data_ptr(), dst.numel(),
                                          _stream_handle(stream)))


def mul_mat_glu(up_name: str, up_ne, gate_name: str, gate_ne, x, dst, stream=None) -> bool:
    """ggml_cuda_q4rdna_mul_mat_glu (SWIGLU only): dst = (W_up x) * silu(W_gate x)."""
    return bool(_lib().q4rdna_mul_mat_glu(up_name.encode(), up_ne[0], up_ne[1], gate_name.encode(), gate_ne[0],
                                          gate_ne[1], x.data_ptr(), x.numel(), dst.data_ptr(), dst.numel(),
                                          _stream_handle(stream)))


def registry_hits(weight_name: str) -> int:
    return int(_lib().q4rdna_registry_hits(weight_name.encode()))


def registry_reset() -> None:
    _lib().q4rdna_registry_reset()


def report_stats() -> None:
    _lib().q4rdna_report_stats()


def kernel_name(B: int = 1) -> str:
    """Name of the GEMV kernel the library launches for batch B: the CTA-split
    int8 kernel for B = 1..2, the mma.sync tile path for B = 3..7, the tcgen05
    tile path (after its activation-prep kernel) for B = 8..16."""
    if B >= 8:
        return "q4::q4_tc_gemv_kernel (+ q4::q4_tc_prep_kernel)"
    return "q4::q4_gemv_mb_kernel" if B >= 3 else "q4::q4_gemv_cta_kernel"
