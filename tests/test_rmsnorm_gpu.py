"""GEMV with a fused RMSNorm producer (q4rdna_gemv_rmsnorm and plan
descriptors with norm_weight) against RMSNorm in fp64 followed by the fp64
oracle GEMV.  ggml's definition: h / sqrt(mean(h^2) + eps) * g.  The tolerance
is tests/tolerance.py's, applied to the normalised input.  Needs a B200."""
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
EPS = 1e-6


def to_dev(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def inputs(K, B, seed):
    rng = np.random.default_rng(seed)
    h = (rng.standard_normal((B, K)) * 3.0).astype(np.float32)
    g = (1.0 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    return h, g


def normed(h, g, eps=EPS):
    h64 = h.astype(np.float64)
    r = 1.0 / np.sqrt(np.mean(h64 * h64, axis=1, keepdims=True) + eps)
    return (h64 * r * g.astype(np.float64)).astype(np.float32)


@pytest.mark.parametrize("B", [1, 2, 4, 8, 16])
@pytest.mark.parametrize("split", [0, 1, 3])
def test_rmsnorm_plain(cuda, B, split):
    N, K = 4096, 4096
    tiles = synth.tiles_np(N, K, 2500 + B)
    h, g = inputs(K, B, 2600 + B + split)
    y = q4rdna.gemv(to_dev(tiles, cuda), to_dev(h, cuda), norm_weight=to_dev(g, cuda), norm_eps=EPS,
                    split=split).cpu().numpy()
    y64, mag = oracle.gemv_f64(tiles, normed(h, g), N, K, threads=THREADS)
    tolerance.check(y, y64, mag, f"rmsnorm B={B} split={split}")


@pytest.mark.parametrize("B,split", [(1, 0), (1, 2), (4, 0), (16, 5)])
def test_rmsnorm_swiglu(cuda, B, split):
    N, K = 12288, 4096
    up, gate = synth.tiles_np(N, K, 2700), synth.tiles_np(N, K, 2701)
    h, g = inputs(K, B, 2702 + B)
    y = q4rdna.gemv(to_dev(up, cuda), to_dev(h, cuda), op=q4rdna.OP_SWIGLU, gate_tiles=to_dev(gate, cuda),
                    norm_weight=to_dev(g, cuda), norm_eps=EPS, split=split).cpu().numpy()
    xn = normed(h, g)
    u64, mu = oracle.gemv_f64(up, xn, N, K, threads=THREADS)
    g64, mg = oracle.gemv_f64(gate, xn, N, K, threads=THREADS)
    silu = g64 / (1.0 + np.exp(-g64))
    tolerance.check(y, u64 * silu, mu * np.abs(silu) + np.abs(u64) * 1.1 * mg, f"rmsnorm swiglu B={B}")


@pytest.mark.parametrize("B", [1, 8])
def test_rmsnorm_add_and_eps(cuda, B):
    N, K = 1024, 4096
    tiles = synth.tiles_np(N, K, 2800)
    h, g = inputs(K, B, 2801)
    h[0] *= 1e-4  # a tiny hidden state: eps matters
    add = synth.x_np(N, B, 2802)
    eps = 1e-2
    y = q4rdna.gemv(to_dev(tiles, cuda), to_dev(h, cuda), op=q4rdna.OP_ADD, add=to_dev(add, cuda),
                    norm_weight=to_dev(g, cuda), norm_eps=eps).cpu().numpy()
    y64, mag = oracle.gemv_f64(tiles, normed(h, g, eps), N, K, threads=THREADS)
    tolerance.check(y, y64 + add, mag + np.abs(add), "rmsnorm add")


@pytest.mark.parametrize("B", [1, 4, 16])
@pytest.mark.parametrize("segments", [1, 0])
def test_rmsnorm_plan_mixed(cuda, B, segments):
    """A plan with a layer's pattern: q/k/v and gate/up read one normed input,
    o and down read plain inputs."""
    K = 1024
    h, g = inputs(K, B, 2900 + B)
    hd, gd = to_dev(h, cuda), to_dev(g, cuda)
    specs = [(2048, "norm", 0), (512, "norm", 0), (4096, "norm", 2), (1024, "plain", 0), (96, "norm", 1)]
    descs, host = [], []
    for i, (N, kind, op) in enumerate(specs):
        t = synth.tiles_np(N, K, 3000 + i)
        gt = synth.tiles_np(N, K, 3010 + i) if op == 2 else None
        a = synth.x_np(N, B, 3020 + i) if op == 1 else None
        x = h if kind == "norm" else synth.x_np(K, B, 3030 + i)
        d = {"tiles": to_dev(t, cuda), "x": hd if kind == "norm" else to_dev(x, cuda),
             "y": torch.empty((B, N), device=cuda), "op": op}
        if kind == "norm":
            d["norm_weight"], d["norm_eps"] = gd, EPS
        if gt is not None:
            d["gate_tiles"] = to_dev(gt, cuda)
        if a is not None:
            d["add"] = to_dev(a, cuda)
        descs.append(d)
        host.append((t, gt, normed(h, g) if kind == "norm" else x, a))
    plan = q4rdna.Plan(descs, B=B)
    plan.set_segments(segments)
    plan.run()
    plan.run()
    for d, (N, kind, op), (t, gt, xn, a) in zip(descs, specs, host):
        y = d["y"].cpu().numpy()
        y64, mag = oracle.gemv_f64(t, xn, N, K, threads=THREADS)
        if op == 0:
            tolerance.check(y, y64, mag, f"plan {kind} {N}")
        elif op == 1:
            tolerance.check(y, y64 + a, mag + np.abs(a), f"plan add {N}")
        else:
            g64, mg = oracle.gemv_f64(gt, xn, N, K, threads=THREADS)
            silu = g64 / (1.0 + np.exp(-g64))
            tolerance.check(y, y64 * silu, mag * np.abs(silu) + np.abs(y64) * 1.1 * mg, f"plan swiglu {N}")
    plan.close()
    assert q4rdna.take_fault() == 0


def test_rmsnorm_errors(cuda):
    import ctypes

    N, K = 1024, 4096
    tiles = to_dev(synth.tiles_np(N, K, 3100), cuda)
    h, g = inputs(K, 1, 3101)
    hd, gd = to_dev(h, cuda), to_dev(g, cuda)
    y = torch.empty(N, device=cuda)
    L = q4rdna.lib
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    args = (tiles.data_ptr(), None, hd.data_ptr())
    assert L.q4rdna_gemv_rmsnorm(*args, None, EPS, None, y.data_ptr(), N, K, 1, 0, None, None, 0, st) == 1
    assert L.q4rdna_gemv_rmsnorm(*args, gd.data_ptr(), -1.0, None, y.data_ptr(), N, K, 1, 0, None, None, 0, st) == 1
    assert L.q4rdna_gemv_rmsnorm(*args, gd.data_ptr() + 4, EPS, None, y.data_ptr(), N, K, 1, 0, None, None, 0,
                                 st) == 3
    assert L.q4rdna_gemv_rmsnorm(*args, gd.data_ptr(), EPS, None, y.data_ptr(), N, K, 1, 7, None, None, 0, st) == 1
    torch.cuda.synchronize()
