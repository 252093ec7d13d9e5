"""The small-batch tile path (B = 3..16) against the CPU oracle: the int8
q4_gemv_mb_kernel, or the f16 q4_gemv_mbh_kernel when the suite runs with
Q4RDNA_TILE=f16 (the library reads it once, at its first launch).  Single calls
over the split range, the add / SwiGLU epilogues, plans, ragged row counts and
extreme activation columns.  Needs a B200."""
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


def to_dev(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


@pytest.mark.parametrize("B", [5, 6, 7, 8, 9, 12, 15, 16])
@pytest.mark.parametrize("N,K", [(1024, 4096), (4096, 12288), (160, 640), (12288, 4096)])
def test_tile_path_batches(cuda, B, N, K):
    tiles = synth.tiles_np(N, K, 1000 + B)
    x = synth.x_np(K, B, 1100 + B)
    y = q4rdna.gemv(to_dev(tiles, cuda), to_dev(x, cuda)).cpu().numpy()
    y64, mag = oracle.gemv_f64(tiles, x, N, K, threads=THREADS)
    tolerance.check(y, y64, mag, f"B={B} {N}x{K}")


@pytest.mark.parametrize("B", [8, 16])
@pytest.mark.parametrize("split", [1, 2, 3, 7, 16])
def test_tile_path_split_sweep(cuda, B, split):
    N, K = 4096, 4096
    tiles = synth.tiles_np(N, K, 1200 + split)
    x = synth.x_np(K, B, 1300 + split)
    y = q4rdna.gemv(to_dev(tiles, cuda), to_dev(x, cuda), split=split).cpu().numpy()
    y64, mag = oracle.gemv_f64(tiles, x, N, K, threads=THREADS)
    tolerance.check(y, y64, mag, f"B={B} split={split}")


def test_tile_path_extreme_columns(cuda):
    """Zero, tiny, huge and mixed-magnitude batch columns: the per-(column,
    group) power-of-two scaling must keep every column in tolerance."""
    N, K, B = 1024, 4096, 16
    tiles = synth.tiles_np(N, K, 1400)
    x = synth.x_np(K, B, 1401)
    x[1] = 0.0
    x[2] *= 1e-30
    x[3] *= 1e30
    x[4, ::2] *= 1e-6          # tiny and normal values inside one group
    x[5, :64] = 0.0            # one all-zero group
    x[6] = np.float32(1e-40)   # f32 subnormal activations: below the 2^-104 range, flushed
    y = q4rdna.gemv(to_dev(tiles, cuda), to_dev(x, cuda)).cpu().numpy()
    y64, mag = oracle.gemv_f64(tiles, x, N, K, threads=THREADS)
    assert np.all(y[1] == 0.0)
    assert np.all(np.isfinite(y[6])) and np.max(np.abs(y[6])) <= 1e-36
    for b in range(B):
        if b in (1, 6):
            continue
        tolerance.check(y[b], y64[b], mag[b], f"column {b}")


@pytest.mark.parametrize("B,split", [(8, 0), (16, 1), (11, 5)])
def test_tile_path_add(cuda, B, split):
    N, K = 4096, 4096
    tiles = synth.tiles_np(N, K, 1500)
    x = synth.x_np(K, B, 1501)
    add = synth.x_np(N, B, 1502)
    y = q4rdna.gemv(to_dev(tiles, cuda), to_dev(x, cuda), op=q4rdna.OP_ADD, add=to_dev(add, cuda),
                    split=split).cpu().numpy()
    y64, mag = oracle.gemv_f64(tiles, x, N, K, threads=THREADS)
    tolerance.check(y, y64 + add, mag + np.abs(add), f"add B={B}")


@pytest.mark.parametrize("N,K,B,split", [(12288, 4096, 8, 0), (12288, 4096, 16, 1), (1024, 4096, 16, 3),
                                         (96, 128, 9, 0)])
def test_tile_path_swiglu(cuda, N, K, B, split):
    up, gate = synth.tiles_np(N, K, 1600), synth.tiles_np(N, K, 1601)
    x = synth.x_np(K, B, 1602)
    y = q4rdna.gemv(to_dev(up, cuda), to_dev(x, cuda), op=q4rdna.OP_SWIGLU, gate_tiles=to_dev(gate, cuda),
                    split=split).cpu().numpy()
    u64, mu = oracle.gemv_f64(up, x, N, K, threads=THREADS)
    g64, mg = oracle.gemv_f64(gate, x, N, K, threads=THREADS)
    silu = g64 / (1.0 + np.exp(-g64))
    mag = mu * np.abs(silu) + np.abs(u64) * 1.1 * mg
    tolerance.check(y, u64 * silu, mag, f"swiglu B={B}")


@pytest.mark.parametrize("B", [8, 16])
def test_tile_path_plan(cuda, B):
    specs = [(4096, 4096, 0), (1024, 4096, 0), (12288, 4096, 2), (4096, 12288, 1), (96, 128, 0)]
    descs, host = [], []
    for i, (N, K, op) in enumerate(specs):
        t = synth.tiles_np(N, K, 1700 + i)
        g = synth.tiles_np(N, K, 1710 + i) if op == 2 else None
        x = synth.x_np(K, B, 1720 + i)
        a = synth.x_np(N, B, 1730 + i) if op == 1 else None
        d = {"tiles": to_dev(t, cuda), "x": to_dev(x, cuda), "y": torch.empty((B, N), device=cuda), "op": op}
        if g is not None:
            d["gate_tiles"] = to_dev(g, cuda)
        if a is not None:
            d["add"] = to_dev(a, cuda)
        descs.append(d)
        host.append((t, g, x, a))
    plan = q4rdna.Plan(descs, B=B)
    plan.run()
    first = [d["y"].cpu().numpy().copy() for d in descs]
    plan.run()
    for d, f, (N, K, op), (t, g, x, a) in zip(descs, first, specs, host):
        y = d["y"].cpu().numpy()
        assert np.array_equal(y.view(np.uint32), f.view(np.uint32)), "plan runs differ"
        y64, mag = oracle.gemv_f64(t, x, N, K, threads=THREADS)
        if op == 0:
            tolerance.check(y, y64, mag, f"plan B={B} {N}x{K}")
        elif op == 1:
            tolerance.check(y, y64 + a, mag + np.abs(a), f"plan add B={B}")
        else:
            g64, mg = oracle.gemv_f64(g, x, N, K, threads=THREADS)
            silu = g64 / (1.0 + np.exp(-g64))
            tolerance.check(y, y64 * silu, mag * np.abs(silu) + np.abs(y64) * 1.1 * mg, f"plan swiglu B={B}")
    plan.close()
    assert q4rdna.take_fault() == 0


@pytest.mark.parametrize("B", [1, 4])
def test_batch1_kernel_extreme_columns(cuda, B):
    """The batch-1 kernels take the same activation range."""
    N, K = 1024, 4096
    tiles = synth.tiles_np(N, K, 1410)
    x = synth.x_np(K, B, 1411)
    x[0] *= 1e-30 if B == 1 else 1.0
    if B == 4:
        x[1] *= 1e-30
        x[2] *= 1e30
        x[3, 64:128] = 0.0
    y = q4rdna.gemv(to_dev(tiles, cuda), to_dev(x, cuda)).cpu().numpy()
    y64, mag = oracle.gemv_f64(tiles, x, N, K, threads=THREADS)
    for b in range(B):
        tolerance.check(y[b], y64[b], mag[b], f"column {b}")


def test_tile_path_matches_columnwise_batch1(cuda):
    """Each column of a B = 16 call equals, within tolerance, the same column
    run alone, and the batch-1 and tile paths agree with each other."""
    N, K, B = 4096, 4096, 16
    tiles = to_dev(synth.tiles_np(N, K, 1800), cuda)
    x = synth.x_np(K, B, 1801)
    yb = q4rdna.gemv(tiles, to_dev(x, cuda)).cpu().numpy()
    for b in (0, 7, 15):
        y1 = q4rdna.gemv(tiles, to_dev(x[b:b + 1], cuda)).cpu().numpy()[0]
        assert np.linalg.norm(yb[b] - y1) / np.linalg.norm(y1) <= 2e-6
