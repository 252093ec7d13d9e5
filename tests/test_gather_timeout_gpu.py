"""The fused gather's bounded flag wait runs out, on one GPU.  Needs a B200.

A plan gathers over world = 2, but both "ranks'" buffers and flag arrays are
local allocations and rank 1 never runs: its flag at rank 0 is never raised.
The signal kernel's wait must give up after the plan's timeout, set bit 1 of
q4rdna_take_fault and return, so the stream completes and the context stays
usable.  Then the missing flag is raised by hand (as if the peer had arrived)
and the next run must report no fault.  No GPU fault is involved: the wait is
a polling loop with an iteration limit.
"""
import ctypes
import time

import numpy as np
import torch
import pytest

import oracle
import q4rdna
import tolerance
from q4rdna import synth

pytestmark = pytest.mark.gpu


def test_gather_flag_wait_times_out_and_recovers(cuda):
    L = q4rdna.lib
    N, K, B = 1024, 4096, 1
    tiles = synth.tiles_np(N, K, 9100)
    x = synth.x_np(K, B, 9101)
    td = torch.from_numpy(tiles).to(cuda)
    xd = torch.from_numpy(x).to(cuda)
    y = torch.zeros((B, N), dtype=torch.float32, device=cuda)
    plan = q4rdna.Plan([{"tiles": td, "x": xd, "y": y}], B=B)
    world, rank, nrank = 2, 0, B * N
    g0 = [torch.zeros(world * nrank, device=cuda) for _ in range(world)]
    g1 = [torch.zeros(world * nrank, device=cuda) for _ in range(world)]
    flags = [torch.zeros(64, dtype=torch.int32, device=cuda) for _ in range(world)]
    arr = lambda ts: (ctypes.c_void_p * world)(*[t.data_ptr() for t in ts])  # noqa: E731
    q4rdna.check(L.q4rdna_plan_set_gather_timeout(plan._h, 2000), "set_gather_timeout")  # ~2 ms
    q4rdna.check(L.q4rdna_plan_set_gather(plan._h, world, rank, y.data_ptr(), nrank, arr(g0), arr(g1), arr(flags)),
                 "set_gather")
    assert q4rdna.take_fault() == 0

    # run 1: rank 1's flag never arrives -> the wait expires
    t0 = time.perf_counter()
    plan.run()
    torch.cuda.synchronize()
    took = time.perf_counter() - t0
    fault = q4rdna.take_fault()
    assert fault & 2, f"fault flags {fault:#x}: the gather wait did not report its expiry"
    assert took < 5.0, f"the expired wait took {took:.1f} s"
    assert L.q4rdna_plan_gather_parity(plan._h) == 1
    # this rank's own outputs are complete, here and in its slice of both "ranks'" buffer 1
    y64, mag = oracle.gemv_f64(tiles, x, N, K, threads=8)
    yv = y.cpu().numpy()
    tolerance.check(yv, y64, mag, "gather run with an absent peer")
    for p in range(world):
        assert np.array_equal(g1[p][:nrank].cpu().numpy().view(np.uint32), yv.reshape(-1).view(np.uint32))
    # this rank raised its own flag at both "ranks" for run 1
    assert int(flags[0][rank]) == 1 and int(flags[1][rank]) == 1

    # the peer "arrives": its flag at rank 0 is raised past the next run's epoch
    flags[0][1] = 1000
    torch.cuda.synchronize()
    plan.run()
    torch.cuda.synchronize()
    assert q4rdna.take_fault() == 0
    assert L.q4rdna_plan_gather_parity(plan._h) == 0
    for p in range(world):
        assert np.array_equal(g0[p][:nrank].cpu().numpy().view(np.uint32), yv.reshape(-1).view(np.uint32))
    plan.close()


def test_run_host_with_gather_on_local_buffers(cuda):
    """q4rdna_plan_run_host on a gather plan: the activations come from pinned
    host memory, every output lands in y, in this rank's slice of both "ranks'"
    gathered buffer (parity alternating per run) and in the host buffer, and
    the flag exchange closes each run.  The absent peer's flag at this rank is
    raised in advance, so no wait expires."""
    L = q4rdna.lib
    B = 2
    shapes = [(4096, 4096), (1024, 4096), (4096, 12288)]
    xs = [synth.x_np(K, B, 9300 + i) for i, (_, K) in enumerate(shapes)]
    tiles = [synth.tiles_np(N, K, 9200 + i) for i, (N, K) in enumerate(shapes)]
    x_all = torch.from_numpy(np.concatenate([x.reshape(-1) for x in xs])).to(cuda)
    nrank = sum(B * N for N, _ in shapes)
    y_all = torch.zeros(nrank, dtype=torch.float32, device=cuda)
    descs, xo, yo = [], 0, 0
    for (N, K), t in zip(shapes, tiles):
        descs.append({"tiles": torch.from_numpy(t).to(cuda), "x": x_all[xo:xo + B * K].view(B, K),
                      "y": y_all[yo:yo + B * N].view(B, N)})
        xo += B * K
        yo += B * N
    plan = q4rdna.Plan(descs, B=B)
    world, rank = 2, 0
    g0 = [torch.zeros(world * nrank, device=cuda) for _ in range(world)]
    g1 = [torch.zeros(world * nrank, device=cuda) for _ in range(world)]
    flags = [torch.zeros(64, dtype=torch.int32, device=cuda) for _ in range(world)]
    flags[0][1] = 1 << 20  # the peer has "arrived" for every run of this test
    arr = lambda ts: (ctypes.c_void_p * world)(*[t.data_ptr() for t in ts])  # noqa: E731
    q4rdna.check(L.q4rdna_plan_set_gather(plan._h, world, rank, y_all.data_ptr(), nrank, arr(g0), arr(g1), arr(flags)),
                 "set_gather")
    x_host = x_all.cpu().pin_memory()
    y_host = torch.full((nrank,), float("nan"), dtype=torch.float32).pin_memory()
    x_all.zero_()  # run_host must bring the activations in
    want = []
    for (N, K), t, x in zip(shapes, tiles, xs):
        want.append(oracle.gemv_f64(t, x, N, K, threads=8))
    for run in range(3):
        y_all.fill_(float("nan"))
        plan.run_host(x_host, x_all, y_all, y_host)
        torch.cuda.synchronize()
        assert q4rdna.take_fault() == 0
        par = L.q4rdna_plan_gather_parity(plan._h)
        assert par == (run + 1) % 2
        yv = y_all.cpu().numpy()
        assert np.array_equal(y_host.numpy().view(np.uint32), yv.view(np.uint32))
        g = g1 if par == 1 else g0
        for p in range(world):
            assert np.array_equal(g[p][:nrank].cpu().numpy().view(np.uint32), yv.view(np.uint32))
        off = 0
        for (N, K), (y64, mag) in zip(shapes, want):
            tolerance.check(yv[off:off + B * N].reshape(B, N), y64, mag, f"run_host gather {N}x{K} run {run}")
            off += B * N
    plan.close()


def test_run_many_equals_single_runs(cuda):
    """q4rdna_plan_run_many runs plans in order, as q4rdna_plan_run would."""
    plans, ys, descs = [], [], []
    for i, (N, K) in enumerate([(4096, 4096), (1024, 4096), (4096, 12288)]):
        t = torch.from_numpy(synth.tiles_np(N, K, 9400 + i)).to(cuda)
        x = torch.from_numpy(synth.x_np(K, 1, 9500 + i)).to(cuda)
        y = torch.zeros((1, N), device=cuda)
        plans.append(q4rdna.Plan([{"tiles": t, "x": x, "y": y}], B=1))
        ys.append(y)
        descs.append((t, x))
    for p in plans:
        p.run()
    torch.cuda.synchronize()
    want = [y.cpu().numpy().copy() for y in ys]
    for y in ys:
        y.zero_()
    q4rdna.run_plans(plans)
    torch.cuda.synchronize()
    for y, w in zip(ys, want):
        assert np.array_equal(y.cpu().numpy().view(np.uint32), w.view(np.uint32))
    for p in plans:
        p.close()
