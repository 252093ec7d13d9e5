"""q4rdna_gemv_noalloc: the GEMV for callers that cannot allocate device memory.

An operator hook inside a host framework (the llama.cpp mul_mat hook is the
example) receives only its input and output tensors; the framework owns device
memory, and a cudaMalloc there would stall the device and escape the
framework's memory accounting.  This entry point takes no workspace: its
split-K scratch is a fixed 8 MiB array inside the library.  These tests call it
through the C ABI, compare it with q4rdna_gemv (the workspace entry point) on
two calls in a row, and check the size limit.  This file is collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
import q4rdna
import tolerance
from q4rdna import synth

pytestmark = pytest.mark.gpu


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _with_workspace(td, xd, N, K, B):
    """Reference result: the existing entry point with a caller-owned workspace."""
    L = q4rdna.lib
    need = L.q4rdna_workspace_bytes(N, K, B, q4rdna.OP_PLAIN, None)
    ws = torch.zeros(max(need, 1), dtype=torch.uint8, device=td.device)
    y = torch.empty((B, N), dtype=torch.float32, device=td.device)
    assert L.q4rdna_gemv(td.data_ptr(), xd.data_ptr(), y.data_ptr(), N, K, B, None,
                         ws.data_ptr() if need else None, need, _stream()) == q4rdna.OK
    return y


def _no_alloc(td, xd, N, K, B):
    y = torch.full((B, N), float("nan"), dtype=torch.float32, device=td.device)
    assert q4rdna.lib.q4rdna_gemv_noalloc(td.data_ptr(), xd.data_ptr(), y.data_ptr(), N, K, B, None,
                                          _stream()) == q4rdna.OK
    return y


def test_no_alloc_matches_workspace_entry_point_on_two_calls(cuda):
    # Two calls in a row share the scratch: the second (a different shape, with
    # more row blocks) must not see the first call's partial sums.
    # Single calls at B <= 2 whose K-ranges meet in a thread-block cluster need
    # no scratch at all; B = 8 (the tensor-core path) always uses it, for the
    # prepared activation, so the last two calls exercise the shared array.
    cases = [(4096, 12288, 1, 11), (12288, 4096, 2, 12), (12288, 4096, 8, 13), (4096, 4096, 8, 14)]
    used = [q4rdna.lib.q4rdna_workspace_bytes(N, K, B, q4rdna.OP_PLAIN, None) for N, K, B, _ in cases]
    assert used[2] > 0 and used[3] > 0
    for N, K, B, seed in cases:
        tiles = synth.tiles_np(N, K, seed)
        x = synth.x_np(K, B, seed + 100)
        td = torch.from_numpy(tiles).to(cuda)
        xd = torch.from_numpy(x).to(cuda)
        y_ref = _with_workspace(td, xd, N, K, B).cpu().numpy()
        y = _no_alloc(td, xd, N, K, B).cpu().numpy()
        y64, mag = oracle.gemv_f64(tiles, x, N, K, threads=8)
        tolerance.check(y, y64, mag, f"no-alloc vs fp64 oracle {N}x{K} B={B}")
        # and bit for bit what the workspace entry point computes with the same split
        assert np.array_equal(y.view(np.uint32), y_ref.view(np.uint32))


def test_no_alloc_rejects_scratch_beyond_its_limit(cuda):
    L = q4rdna.lib
    cfg = q4rdna.Cfg()
    cfg.split = 64
    N, K = 65536, 4096  # 64 splits x 65536 rows x 4 B = 16 MiB of partials > 8 MiB
    assert L.q4rdna_workspace_bytes(N, K, 1, q4rdna.OP_PLAIN, ctypes.byref(cfg)) > (8 << 20)
    dummy = torch.empty(256, dtype=torch.uint8, device=cuda)
    assert L.q4rdna_gemv_noalloc(dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), N, K, 1,
                                 ctypes.byref(cfg), _stream()) == 11  # Q4RDNA_ERR_TOO_LARGE
    assert L.q4rdna_gemv_noalloc(None, dummy.data_ptr(), dummy.data_ptr(), 32, 64, 1, None, _stream()) == 1
