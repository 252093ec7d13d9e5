"""ctypes loader for the CPU oracle.  TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import this
package, and only as the checker or as the timed CPU baseline.  The product
library never imports or links it.

``lib`` is the C restatement (q4rdna_oracle.c).

fp16 scale decoding has two modes (keyword ``decode``):
  "ieee"   - IEEE binary16, what the reference GPU kernel computes
             (__half2float, source/q4rdna.cu:370); the default, used as the
             parity target of the CUDA path;
  "refcpu" - the reference CPU tools' decoder, which halves fp16 subnormals
             (q4rdna_cpu_experiment.cpp:53); bit-exact with the reference's
             CPU GEMV (q4rdna_gemv_bench.hip:189-211).
Both agree on every normal, zero, inf and NaN pattern.  ``ref`` is the reference's own
CPU code compiled from its sources (oracle/_ref/libq4ref.so), or None where it
was not built.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_u8p = ctypes.POINTER(ctypes.c_uint8)
_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_i64 = ctypes.c_int64


def _load(path):
    return ctypes.CDLL(path) if os.path.exists(path) else None


lib = _load(os.path.join(_HERE, "liboracle.so"))
ref = _load(os.path.join(_HERE, "_ref", "libq4ref.so"))
REF_PACK_BIN = os.path.join(_HERE, "_ref", "q4rdna_sidecar_pack")

if lib is not None:
    lib.q4o_fp16_to_f32.argtypes = [ctypes.c_uint16]
    lib.q4o_fp16_to_f32.restype = ctypes.c_float
    lib.q4o_f32_to_fp16.argtypes = [ctypes.c_float]
    lib.q4o_f32_to_fp16.restype = ctypes.c_uint16
    lib.q4o_fp16_to_f32_ieee.argtypes = [ctypes.c_uint16]
    lib.q4o_fp16_to_f32_ieee.restype = ctypes.c_float
    _ci = ctypes.c_int
    lib.q4o_dequant.argtypes = [_u8p, _i64, _i64, _f32p, _ci]
    lib.q4o_gemv_f32.argtypes = [_u8p, _f32p, _f32p, _i64, _i64, _i64, _ci, _ci]
    lib.q4o_gemv_f64.argtypes = [_u8p, _f32p, _f64p, _f64p, _i64, _i64, _i64, _ci, _ci]
    lib.q4o_gemv_add_f32.argtypes = [_u8p, _f32p, _f32p, _f32p, _i64, _i64, _i64, _ci, _ci]
    lib.q4o_gemv_swiglu_f32.argtypes = [_u8p, _u8p, _f32p, _f32p, _f32p, _i64, _i64, _i64, _ci, _ci]
    lib.q4o_select_scale.argtypes = [_f32p]
    lib.q4o_select_scale.restype = ctypes.c_uint16
    lib.q4o_pack_bf16.argtypes = [_u16p, _i64, _i64, _u8p, ctypes.c_int]
    lib.q4o_q4k_dequant.argtypes = [_u8p, _i64, _i64, _f32p, _ci]
    lib.q4o_q4k_gemv_f32.argtypes = [_u8p, _f32p, _f32p, _i64, _i64, _i64, _ci, _ci]
    lib.q4o_q4k_gemv_f64.argtypes = [_u8p, _f32p, _f64p, _f64p, _i64, _i64, _i64, _ci, _ci]
    lib.q4o_silu.argtypes = [ctypes.c_float]
    lib.q4o_silu.restype = ctypes.c_float

if ref is not None:
    ref.q4ref_bench_rows.restype = ctypes.c_int
    ref.q4ref_bench_columns.restype = ctypes.c_int
    ref.q4ref_bench_half_to_float.argtypes = [ctypes.c_uint16]
    ref.q4ref_bench_half_to_float.restype = ctypes.c_float
    ref.q4ref_bench_gemv.argtypes = [_u8p, ctypes.c_uint64, _f32p, _f32p]
    ref.q4ref_bench_gemv.restype = ctypes.c_int
    ref.q4ref_bench_prepare.argtypes = [_u8p, ctypes.c_uint64]
    ref.q4ref_bench_prepare.restype = ctypes.c_void_p
    ref.q4ref_bench_run.argtypes = [ctypes.c_void_p, _f32p, _f32p]
    ref.q4ref_bench_run.restype = ctypes.c_int
    ref.q4ref_bench_release.argtypes = [ctypes.c_void_p]
    ref.q4ref_pack_select_scale.argtypes = [_f32p]
    ref.q4ref_pack_select_scale.restype = ctypes.c_uint16
    ref.q4ref_pack_float_to_fp16.argtypes = [ctypes.c_float]
    ref.q4ref_pack_float_to_fp16.restype = ctypes.c_uint16
    ref.q4ref_pack_fp16_to_float.argtypes = [ctypes.c_uint16]
    ref.q4ref_pack_fp16_to_float.restype = ctypes.c_float
    ref.q4ref_exp_float_to_fp16.argtypes = [ctypes.c_float]
    ref.q4ref_exp_float_to_fp16.restype = ctypes.c_uint16
    ref.q4ref_exp_fp16_to_float.argtypes = [ctypes.c_uint16]
    ref.q4ref_exp_fp16_to_float.restype = ctypes.c_float
    ref.q4ref_exp_dequant_q4k.argtypes = [_u8p, ctypes.c_uint64, _f32p]


def _need():
    if lib is None:
        raise RuntimeError("oracle/liboracle.so is not built (run `make -C oracle`)")


def _mode(decode):
    if decode not in ("ieee", "refcpu"):
        raise ValueError(f"decode must be 'ieee' or 'refcpu', not {decode!r}")
    return 1 if decode == "ieee" else 0


def _p(a, t):
    return a.ctypes.data_as(t)


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def gemv_f32(tiles, x, N, K, threads=1, decode="ieee"):
    """Reference-order f32 GEMV.  x: [B, K] (or [K]); returns [B, N] (or [N])."""
    _need()
    t = _c(tiles, np.uint8).reshape(-1)
    xv = _c(x, np.float32)
    squeeze = xv.ndim == 1
    xv = xv.reshape(-1, K)
    B = xv.shape[0]
    y = np.empty((B, N), np.float32)
    lib.q4o_gemv_f32(_p(t, _u8p), _p(xv, _f32p), _p(y, _f32p), N, K, B, threads, _mode(decode))
    return y[0] if squeeze else y


def gemv_f64(tiles, x, N, K, threads=1, decode="ieee"):
    """fp64-accumulated y and per-row sum |W x|; shapes as gemv_f32."""
    _need()
    t = _c(tiles, np.uint8).reshape(-1)
    xv = _c(x, np.float32)
    squeeze = xv.ndim == 1
    xv = xv.reshape(-1, K)
    B = xv.shape[0]
    y = np.empty((B, N), np.float64)
    mag = np.empty((B, N), np.float64)
    lib.q4o_gemv_f64(_p(t, _u8p), _p(xv, _f32p), _p(y, _f64p), _p(mag, _f64p), N, K, B, threads, _mode(decode))
    return (y[0], mag[0]) if squeeze else (y, mag)


def gemv_add_f32(tiles, x, add, N, K, threads=1, decode="ieee"):
    _need()
    t = _c(tiles, np.uint8).reshape(-1)
    xv = _c(x, np.float32).reshape(-1, K)
    B = xv.shape[0]
    a = _c(add, np.float32).reshape(B, N)
    y = np.empty((B, N), np.float32)
    lib.q4o_gemv_add_f32(_p(t, _u8p), _p(xv, _f32p), _p(a, _f32p), _p(y, _f32p), N, K, B, threads, _mode(decode))
    return y


def gemv_swiglu_f32(up, gate, x, N, K, threads=1, decode="ieee"):
    _need()
    u = _c(up, np.uint8).reshape(-1)
    g = _c(gate, np.uint8).reshape(-1)
    xv = _c(x, np.float32).reshape(-1, K)
    B = xv.shape[0]
    y = np.empty((B, N), np.float32)
    scratch = np.empty((B, N), np.float32)
    lib.q4o_gemv_swiglu_f32(_p(u, _u8p), _p(g, _u8p), _p(xv, _f32p), _p(y, _f32p),
                            _p(scratch, _f32p), N, K, B, threads, _mode(decode))
    return y


def dequant(tiles, N, K, decode="ieee"):
    _need()
    t = _c(tiles, np.uint8).reshape(-1)
    W = np.empty((N, K), np.float32)
    lib.q4o_dequant(_p(t, _u8p), N, K, _p(W, _f32p), _mode(decode))
    return W


def q4k_dequant(blocks, N, K, decode="ieee"):
    """Q4_K rows -> dense f32 W[N, K] (q4rdna_cpu_experiment.cpp:112-135)."""
    _need()
    t = _c(blocks, np.uint8).reshape(-1)
    W = np.empty((N, K), np.float32)
    lib.q4o_q4k_dequant(_p(t, _u8p), N, K, _p(W, _f32p), _mode(decode))
    return W


def q4k_gemv_f32(blocks, x, N, K, threads=1, decode="ieee"):
    """The reference Q4_K kernel's f32 order (q4rdna_gemv_bench.hip:93-135).
    x: [B, K]; returns [B, N]."""
    _need()
    t = _c(blocks, np.uint8).reshape(-1)
    xv = _c(x, np.float32).reshape(-1, K)
    B = xv.shape[0]
    y = np.empty((B, N), np.float32)
    lib.q4o_q4k_gemv_f32(_p(t, _u8p), _p(xv, _f32p), _p(y, _f32p), N, K, B, threads, _mode(decode))
    return y


def q4k_gemv_f64(blocks, x, N, K, threads=1, decode="ieee"):
    """fp64-accumulated y over the dequantised Q4_K weights, and sum |W x|."""
    _need()
    t = _c(blocks, np.uint8).reshape(-1)
    xv = _c(x, np.float32).reshape(-1, K)
    B = xv.shape[0]
    y = np.empty((B, N), np.float64)
    mag = np.empty((B, N), np.float64)
    lib.q4o_q4k_gemv_f64(_p(t, _u8p), _p(xv, _f32p), _p(y, _f64p), _p(mag, _f64p), N, K, B, threads, _mode(decode))
    return y, mag


def ref_q4k_dequant(blocks):
    """The reference's own dequantize_q4_k over consecutive blocks (compiled
    from q4rdna_cpu_experiment.cpp where it lies) -> f32 [nblocks * 256]."""
    if ref is None:
        raise RuntimeError("oracle/_ref/libq4ref.so is not built")
    t = _c(blocks, np.uint8).reshape(-1)
    n = t.size // 144
    out = np.empty(n * 256, np.float32)
    ref.q4ref_exp_dequant_q4k(_p(t, _u8p), n, _p(out, _f32p))
    return out


def pack_bf16(bf16, threads=1):
    """bf16 bit patterns [N, K] (uint16) -> tiles (uint8, N*K*34/64 bytes)."""
    _need()
    b = _c(bf16, np.uint16)
    N, K = b.shape
    tiles = np.zeros(N * K * 34 // 64, np.uint8)
    lib.q4o_pack_bf16(_p(b, _u16p), N, K, _p(tiles, _u8p), threads)
    return tiles


def select_scale(v64):
    _need()
    v = _c(v64, np.float32)
    return int(lib.q4o_select_scale(_p(v, _f32p)))


def ref_bench_gemv(tiles, x):
    """The reference's own CPU GEMV (fixed 12288 x 4096), or None if not built."""
    if ref is None:
        return None
    t = _c(tiles, np.uint8).reshape(-1)
    xv = _c(x, np.float32).reshape(-1)
    y = np.empty(ref.q4ref_bench_rows(), np.float32)
    rc = ref.q4ref_bench_gemv(_p(t, _u8p), t.size, _p(xv, _f32p), _p(y, _f32p))
    if rc != 0:
        raise ValueError("reference bench GEMV needs a 12288 x 4096 tile buffer")
    return y


class RefBenchGemv:
    """The reference CPU GEMV on one prepared 12288 x 4096 tile buffer, for timing."""

    def __init__(self, tiles):
        if ref is None:
            raise RuntimeError("oracle/_ref not built")
        t = _c(tiles, np.uint8).reshape(-1)
        self._h = ref.q4ref_bench_prepare(_p(t, _u8p), t.size)
        if not self._h:
            raise ValueError("reference bench GEMV needs a 12288 x 4096 tile buffer")
        self.y = np.empty(ref.q4ref_bench_rows(), np.float32)

    def __call__(self, x):
        xv = _c(x, np.float32).reshape(-1)
        ref.q4ref_bench_run(self._h, _p(xv, _f32p), _p(self.y, _f32p))
        return self.y

    def __del__(self):
        if getattr(self, "_h", None):
            ref.q4ref_bench_release(self._h)
            self._h = None
