"""q4rdna_plan_run_host: a plan run from pinned host buffers, with the copies
overlapped segment by segment, must give exactly the outputs of copy-in,
q4rdna_plan_run, copy-out.  Needs a B200."""
import numpy as np
import pytest
import torch

import q4rdna
from q4rdna import synth, tp

pytestmark = pytest.mark.gpu

TENSORS = [("blk.0.attn_q.weight", 4096, 4096), ("blk.0.attn_k.weight", 1024, 4096),
           ("blk.0.ffn_gate.weight", 12288, 4096), ("blk.0.ffn_down.weight", 4096, 12288),
           ("blk.1.attn_v.weight", 96, 128), ("blk.1.attn_o.weight", 4096, 4096)]


def _step(cuda, B, seed):
    lay = tp.Layout(TENSORS, 1, B)
    x_dev = torch.empty(B * lay.xsz, dtype=torch.float32, device=cuda)
    y_dev = torch.empty(B * lay.ysz, dtype=torch.float32, device=cuda)
    descs, xo = [], 0
    for i, s in enumerate(lay.slots):
        t = torch.from_numpy(synth.tiles_np(s.N, s.K, seed + i)).to(cuda)
        descs.append({"tiles": t, "x": x_dev[B * xo:B * (xo + s.K)].view(B, s.K), "y": lay.local_view(y_dev, i)})
        xo += s.K
    x_host = torch.from_numpy(np.random.default_rng(seed).standard_normal(B * lay.xsz, dtype=np.float32)).pin_memory()
    y_host = torch.empty(B * lay.ysz, dtype=torch.float32).pin_memory()
    return q4rdna.Plan(descs, B=B), x_dev, y_dev, x_host, y_host


@pytest.mark.parametrize("B", [1, 4, 16])
@pytest.mark.parametrize("segments", [0, 1, 3, 6, 50])
def test_run_host_equals_copies_and_run(cuda, B, segments):
    plan, x_dev, y_dev, x_host, y_host = _step(cuda, B, 2000 + B)
    x_dev.copy_(x_host)
    plan.run()
    want = y_dev.cpu().numpy().view(np.uint32).copy()
    x_dev.zero_()
    y_dev.fill_(float("nan"))
    for rep in range(2):  # the second run reuses the plan's segments and events
        y_host.fill_(float("nan"))
        plan.run_host(x_host, x_dev, y_dev, y_host, segments=segments)
        torch.cuda.current_stream().synchronize()
        assert np.array_equal(y_host.numpy().view(np.uint32), want), f"run {rep}"
    plan.close()


def test_run_host_rejects_buffers_not_covering_the_plan(cuda):
    plan, x_dev, y_dev, x_host, y_host = _step(cuda, 1, 2100)
    with pytest.raises(q4rdna.Q4RDNAError):
        plan.run_host(x_host[:-4], x_dev[:-4], y_dev, y_host)
    with pytest.raises(q4rdna.Q4RDNAError):
        plan.run_host(x_host, x_dev, y_dev[4:], y_host[4:])
    plan.close()


def test_run_host_rejects_overlapping_segments(cuda):
    """Two descriptors reading the same activations in different segments
    cannot be overlapped safely: the call refuses instead of racing."""
    N, K = 1024, 4096
    x_dev = torch.empty(K, dtype=torch.float32, device=cuda)
    y_dev = torch.empty(2 * N, dtype=torch.float32, device=cuda)
    descs = [{"tiles": torch.from_numpy(synth.tiles_np(N, K, 2200 + i)).to(cuda), "x": x_dev.view(1, K),
              "y": y_dev[i * N:(i + 1) * N].view(1, N)} for i in range(2)]
    plan = q4rdna.Plan(descs, B=1)
    x_host = torch.zeros(K, dtype=torch.float32).pin_memory()
    y_host = torch.empty(2 * N, dtype=torch.float32).pin_memory()
    with pytest.raises(q4rdna.Q4RDNAError):
        plan.run_host(x_host, x_dev, y_dev, y_host, segments=2)
    plan.run_host(x_host, x_dev, y_dev, y_host, segments=1)  # one segment: nothing overlaps
    torch.cuda.current_stream().synchronize()
    assert np.all(y_host.numpy() == 0.0)
    plan.close()


@pytest.mark.parametrize("B", [1, 8])
@pytest.mark.parametrize("segments", [0, 2, 5, 100])
def test_segmented_run_equals_one_launch(cuda, B, segments):
    plan, x_dev, y_dev, x_host, y_host = _step(cuda, B, 2300 + B)
    x_dev.copy_(x_host)
    plan.run()
    want = y_dev.cpu().numpy().view(np.uint32).copy()
    plan.set_segments(segments)
    for rep in range(2):
        y_dev.fill_(float("nan"))
        plan.run()
        assert np.array_equal(y_dev.cpu().numpy().view(np.uint32), want), f"run {rep}"
    plan.set_segments(1)
    plan.run()
    assert np.array_equal(y_dev.cpu().numpy().view(np.uint32), want)
    plan.close()


@pytest.mark.parametrize("B", [1, 4])
def test_run_host_pageable_output_falls_back_to_copies(cuda, B):
    """Pinned output buffers receive the outputs straight from the kernels; a
    pageable one cannot be mapped for the device, so run_host copies into it
    instead.  Both give exactly the outputs of copy-in, run, copy-out, and a
    change of output buffer between calls is picked up."""
    plan, x_dev, y_dev, x_host, y_pinned = _step(cuda, B, 2400 + B)
    x_dev.copy_(x_host)
    plan.run()
    want = y_dev.cpu().numpy().view(np.uint32).copy()
    y_pageable = torch.empty(y_pinned.numel(), dtype=torch.float32)
    for y_host in (y_pinned, y_pageable, y_pinned):
        y_host.fill_(float("nan"))
        plan.run_host(x_host, x_dev, y_dev, y_host)
        torch.cuda.current_stream().synchronize()
        assert np.array_equal(y_host.numpy().view(np.uint32), want)
        assert np.array_equal(y_dev.cpu().numpy().view(np.uint32), want)
    plan.close()
