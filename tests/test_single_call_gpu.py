"""Single drop-in calls at B = 1..2 (the CTA-split kernel) and their
programmatic dependent launch.  Needs a B200.

q4rdna_gemv at B <= 2 runs one CTA per (128-row block, K-range) with the
K-range split again over the CTA's warps.  With Q4RDNA_CFG_OVERLAP_PREVIOUS a
call may start streaming its weights while the previous kernel on the stream
still runs; it must still read its activation only after that kernel
finished.  A chain of calls in which every call's x is the previous call's y
checks exactly that: it must equal, bit for bit, the same chain launched
without the overlap, and each link must match the fp64 oracle.
"""
import ctypes
import os

import numpy as np
import pytest
import torch

import oracle
import q4rdna
import tolerance
from q4rdna import synth

pytestmark = pytest.mark.gpu
THREADS = max(1, min(16, os.cpu_count() or 1))


def _chain(cuda, tiles_dev, x0, B, overlap, links):
    L = q4rdna.lib
    N = K = 4096
    cfg = q4rdna.Cfg()
    cfg.flags = q4rdna.CFG_OVERLAP_PREVIOUS if overlap else 0
    need = L.q4rdna_workspace_bytes(N, K, B, q4rdna.OP_PLAIN, ctypes.byref(cfg))
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=cuda)
    bufs = [x0.clone(), torch.empty_like(x0)]
    h = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    outs = []
    for i in range(links):
        src, dst = bufs[i % 2], bufs[(i + 1) % 2]
        rc = L.q4rdna_gemv(tiles_dev[i % len(tiles_dev)].data_ptr(), src.data_ptr(), dst.data_ptr(), N, K, B,
                           ctypes.byref(cfg), ws.data_ptr(), need, h)
        assert rc == 0
        if i < 3:
            outs.append(dst.clone())
    torch.cuda.synchronize()
    return bufs[links % 2].cpu().numpy(), [o.cpu().numpy() for o in outs]


@pytest.mark.parametrize("B", [1, 2])
def test_overlapped_chain_matches_plain_chain(cuda, B):
    N = K = 4096
    tiles = [synth.tiles_np(N, K, 7700 + i) for i in range(3)]
    td = [torch.from_numpy(t).to(cuda) for t in tiles]
    x0 = torch.from_numpy(synth.x_np(K, B, 7800)).to(cuda)
    plain, p3 = _chain(cuda, td, x0, B, False, 24)
    over, o3 = _chain(cuda, td, x0, B, True, 24)
    assert np.array_equal(plain.view(np.uint32), over.view(np.uint32))
    # the first links against the fp64 oracle (each on the previous link's f32 output)
    xin = x0.cpu().numpy()
    for i in range(3):
        y64, mag = oracle.gemv_f64(tiles[i], xin, N, K, threads=THREADS)
        tolerance.check(o3[i], y64, mag, f"overlapped link {i} B={B}")
        assert np.array_equal(o3[i].view(np.uint32), p3[i].view(np.uint32))
        xin = o3[i]


@pytest.mark.parametrize("N,K", [(4096, 4096), (12288, 4096), (4096, 12288), (1024, 4096), (160, 640), (96, 64)])
@pytest.mark.parametrize("op", [q4rdna.OP_PLAIN, q4rdna.OP_ADD, q4rdna.OP_SWIGLU])
def test_single_call_ops_with_overlap(cuda, N, K, op):
    """Every epilogue through the single-call kernel with the overlap flag, at
    the selector's split and at split 1, against the fp64 oracle."""
    L = q4rdna.lib
    tiles = synth.tiles_np(N, K, 7900 + N + K)
    gate = synth.tiles_np(N, K, 7950 + N + K)
    x = synth.x_np(K, 1, 7990 + K)
    add = synth.x_np(N, 1, 7995 + N)
    td, gd = torch.from_numpy(tiles).to(cuda), torch.from_numpy(gate).to(cuda)
    xd, ad = torch.from_numpy(x).to(cuda), torch.from_numpy(add).to(cuda)
    y64, mag = oracle.gemv_f64(tiles, x, N, K, threads=THREADS)
    for split in (0, 1):
        cfg = q4rdna.Cfg()
        cfg.split = split
        cfg.flags = q4rdna.CFG_OVERLAP_PREVIOUS
        need = L.q4rdna_workspace_bytes(N, K, 1, op, ctypes.byref(cfg))
        ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=cuda)
        y = torch.full((1, N), float("nan"), device=cuda)
        h = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        if op == q4rdna.OP_PLAIN:
            rc = L.q4rdna_gemv(td.data_ptr(), xd.data_ptr(), y.data_ptr(), N, K, 1, ctypes.byref(cfg), ws.data_ptr(),
                               need, h)
        elif op == q4rdna.OP_ADD:
            rc = L.q4rdna_gemv_add(td.data_ptr(), xd.data_ptr(), ad.data_ptr(), y.data_ptr(), N, K, 1,
                                   ctypes.byref(cfg), ws.data_ptr(), need, h)
        else:
            rc = L.q4rdna_gemv_swiglu(td.data_ptr(), gd.data_ptr(), xd.data_ptr(), y.data_ptr(), N, K, 1,
                                      ctypes.byref(cfg), ws.data_ptr(), need, h)
        assert rc == 0
        yv = y.cpu().numpy()
        what = f"{N}x{K} op={op} split={split}"
        if op == q4rdna.OP_PLAIN:
            tolerance.check(yv, y64, mag, what)
        elif op == q4rdna.OP_ADD:
            tolerance.check(yv, y64 + add, mag + np.abs(add), what)
        else:
            g64, mg = oracle.gemv_f64(gate, x, N, K, threads=THREADS)
            silu = g64 / (1.0 + np.exp(-g64))
            tolerance.check(yv, y64 * silu, mag * np.abs(silu) + np.abs(y64) * 1.1 * mg, what)


@pytest.mark.parametrize("B", [1, 2])
@pytest.mark.parametrize("split", [2, 3, 5, 8, 9])
@pytest.mark.parametrize("op", [q4rdna.OP_PLAIN, q4rdna.OP_SWIGLU])
def test_cluster_reduction_matches_plan_reduction(cuda, B, split, op):
    """A single call with 2..8 K-ranges adds them through distributed shared
    memory inside one cluster per row block; a plan (and a single call with
    more than 8) adds them through the workspace after an arrival ticket.
    Both add the same partial sums in the same order, so the outputs must be
    the same bits; and both must match the fp64 oracle.  The fused RMSNorm
    rides along on the plain op."""
    N, K = 1056, 4096  # 9 row blocks, the last one partial
    tiles = synth.tiles_np(N, K, 8100 + split)
    gate = synth.tiles_np(N, K, 8150 + split)
    x = synth.x_np(K, B, 8200 + split)
    g = (np.abs(synth.x_np(K, 1, 8250 + split)[0]) + 0.5).astype(np.float32)
    td, gd = torch.from_numpy(tiles).to(cuda), torch.from_numpy(gate).to(cuda)
    xd, gn = torch.from_numpy(x).to(cuda), torch.from_numpy(g).to(cuda)
    kw = {"op": op, "split": split}
    if op == q4rdna.OP_SWIGLU:
        kw["gate_tiles"] = gd
    norm = {"norm_weight": gn, "norm_eps": 1e-6} if op == q4rdna.OP_PLAIN else {}
    single = q4rdna.gemv(td, xd, **kw, **norm).cpu().numpy()
    y = torch.empty((B, N), device=cuda)
    desc = {"tiles": td, "x": xd, "y": y, "op": op, "split": split}
    if op == q4rdna.OP_SWIGLU:
        desc["gate_tiles"] = gd
    if norm:
        desc.update(norm)
    plan = q4rdna.Plan([desc], B=B)
    plan.run()
    planned = y.cpu().numpy()
    plan.close()
    assert np.array_equal(single.view(np.uint32), planned.view(np.uint32))
    if norm:  # ggml's RMSNorm in fp64: h / sqrt(mean(h^2) + eps) * g
        x64 = x.astype(np.float64)
        xin = (x64 / np.sqrt(np.mean(x64 * x64, axis=1, keepdims=True) + 1e-6) * g.astype(np.float64)).astype(np.float32)
    else:
        xin = x
    y64, mag = oracle.gemv_f64(tiles, xin, N, K, threads=THREADS)
    if op == q4rdna.OP_SWIGLU:
        g64, mg = oracle.gemv_f64(gate, x, N, K, threads=THREADS)
        silu = g64 / (1.0 + np.exp(-g64))
        tolerance.check(single, y64 * silu, mag * np.abs(silu) + np.abs(y64) * 1.1 * mg, f"swiglu split={split}")
    else:
        tolerance.check(single, y64, mag, f"rmsnorm split={split}")
