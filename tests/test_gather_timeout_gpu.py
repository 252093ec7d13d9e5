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
