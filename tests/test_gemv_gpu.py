"""CUDA path vs the CPU oracle (parity tests proper).  Needs a B200.

All calls go through the C ABI (libq4rdna.so via ctypes); torch only owns the
device buffers.  Targets:
  * dequantisation: bit-exact (IEEE fp16 decode, the reference GPU kernel's
    semantics; and bit-exact with the reference CPU code on every tile whose
    scales are not fp16 subnormals);
  * outputs: tests/tolerance.py bounds against the fp64-accumulated oracle.
"""
import os

import numpy as np
import pytest
import torch

import oracle
import q4rdna
import tolerance
from q4rdna import format as fmt, synth

pytestmark = pytest.mark.gpu
THREADS = max(1, min(16, os.cpu_count() or 1))


def to_dev(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def no_subnormal_scales(tiles):
    """Same tiles with every subnormal fp16 scale made normal (exponent bit set)."""
    t = tiles.copy().reshape(-1, fmt.TILE_BYTES)
    s = t[:, :64].copy().view(np.uint16)
    sub = ((s & 0x7C00) == 0) & ((s & 0x03FF) != 0)
    s[sub] |= 0x0400
    t[:, :64] = s.view(np.uint8)
    return t.reshape(-1)


@pytest.mark.parametrize("N,K", [(32, 64), (96, 128), (160, 192), (1024, 4096), (4096, 4096)])
def test_dequant_bit_exact(cuda, N, K):
    tiles = synth.tiles_np(N, K, 1000 + N + K)
    W = q4rdna.dequant(to_dev(tiles, cuda), N, K).cpu().numpy()
    assert np.array_equal(W.view(np.uint32), oracle.dequant(tiles, N, K, decode="ieee").view(np.uint32))
    tn = no_subnormal_scales(tiles)
    Wn = q4rdna.dequant(to_dev(tn, cuda), N, K).cpu().numpy()
    assert np.array_equal(Wn.view(np.uint32), oracle.dequant(tn, N, K, decode="refcpu").view(np.uint32))


SHAPES = [(4096, 4096), (12288, 4096), (4096, 12288), (1024, 4096), (32, 64), (96, 128), (160, 640),
          (224, 1984), (8192, 5120), (5120, 8192)]


@pytest.mark.parametrize("N,K", SHAPES)
def test_gemv_parity_default_split(cuda, N, K):
    tiles = synth.tiles_np(N, K, N * 7 + K)
    x = synth.x_np(K, 1, N + K)
    y = q4rdna.gemv(to_dev(tiles, cuda), to_dev(x, cuda)).cpu().numpy()
    y64, mag = oracle.gemv_f64(tiles, x, N, K, threads=THREADS)
    tolerance.check(y, y64, mag, f"{N}x{K}")


@pytest.mark.parametrize("N,K", [(4096, 12288), (12288, 4096), (1024, 4096)])
@pytest.mark.parametrize("split", list(range(1, 17)))
def test_split_k_sweep(cuda, N, K, split):
    """Config 1: split-K factor 1..16 on the stress shapes; deterministic."""
    tiles = synth.tiles_np(N, K, 3 * N + K)
    x = synth.x_np(K, 1, 17 + split)
    td, xd = to_dev(tiles, cuda), to_dev(x, cuda)
    y1 = q4rdna.gemv(td, xd, split=split).cpu().numpy()
    y2 = q4rdna.gemv(td, xd, split=split).cpu().numpy()
    assert np.array_equal(y1.view(np.uint32), y2.view(np.uint32)), "split-K result not deterministic"
    y64, mag = oracle.gemv_f64(tiles, x, N, K, threads=THREADS)
    tolerance.check(y1, y64, mag, f"{N}x{K} split={split}")


def test_reference_cpu_gemv_on_normal_scales(cuda):
    """Against the reference's own CPU GEMV order and decoder (oracle refcpu mode,
    bit-exact with q4rdna_gemv_bench.hip:189-211), on tiles without subnormal
    scales, with the bench's sin/cos activation (q4rdna_gemv_bench.hip:224-227)."""
    N, K = 12288, 4096
    tiles = no_subnormal_scales(synth.tiles_np(N, K, 20260816))
    i = np.arange(K, dtype=np.float32)
    x = (np.sin(i * np.float32(0.013)) * np.float32(0.25) + np.cos(i * np.float32(0.007)) * np.float32(0.125)).astype(np.float32)
    y = q4rdna.gemv(to_dev(tiles, cuda), to_dev(x, cuda)).cpu().numpy()
    yref = oracle.gemv_f32(tiles, x, N, K, threads=THREADS, decode="refcpu")
    y64, mag = oracle.gemv_f64(tiles, x, N, K, threads=THREADS, decode="refcpu")
    assert np.linalg.norm(y - yref) / np.linalg.norm(yref) <= 1e-5  # the reference bench's own check
    tolerance.check(y, y64, mag, "bench sin/cos")


@pytest.mark.parametrize("B", [1, 2, 3, 4, 5, 8, 16])
@pytest.mark.parametrize("N,K", [(1024, 4096), (160, 640)])
def test_batch(cuda, B, N, K):
    tiles = synth.tiles_np(N, K, 40 + B)
    x = synth.x_np(K, B, 50 + B)
    y = q4rdna.gemv(to_dev(tiles, cuda), to_dev(x, cuda)).cpu().numpy()
    y64, mag = oracle.gemv_f64(tiles, x, N, K, threads=THREADS)
    tolerance.check(y, y64, mag, f"B={B}")


@pytest.mark.parametrize("split", [0, 1, 5])
def test_add_epilogue(cuda, split):
    N, K, B = 4096, 4096, 2
    tiles = synth.tiles_np(N, K, 61)
    x = synth.x_np(K, B, 62)
    add = synth.x_np(N, B, 63)
    y = q4rdna.gemv(to_dev(tiles, cuda), to_dev(x, cuda), op=q4rdna.OP_ADD, add=to_dev(add, cuda),
                    split=split).cpu().numpy()
    y64, mag = oracle.gemv_f64(tiles, x, N, K, threads=THREADS)
    tolerance.check(y, y64 + add, mag + np.abs(add), "add")


@pytest.mark.parametrize("N,K,split", [(12288, 4096, 0), (12288, 4096, 1), (1024, 4096, 3), (96, 128, 0)])
def test_swiglu_epilogue(cuda, N, K, split):
    up, gate = synth.tiles_np(N, K, 71), synth.tiles_np(N, K, 72)
    x = synth.x_np(K, 1, 73)
    y = q4rdna.gemv(to_dev(up, cuda), to_dev(x, cuda), op=q4rdna.OP_SWIGLU, gate_tiles=to_dev(gate, cuda),
                    split=split).cpu().numpy()
    u64, mu = oracle.gemv_f64(up, x, N, K, threads=THREADS)
    g64, mg = oracle.gemv_f64(gate, x, N, K, threads=THREADS)
    sig = 1.0 / (1.0 + np.exp(-g64))
    silu = g64 * sig
    y64 = u64 * silu
    # first-order bound: |d(u*silu(g))| <= |silu(g)| du + |u| |silu'(g)| dg, |silu'| <= 1.1
    mag = mu * np.abs(silu) + np.abs(u64) * 1.1 * mg
    tolerance.check(y, y64, mag, "swiglu")
    # the oracle's f32 SwiGLU (reference order) agrees too
    yo = oracle.gemv_swiglu_f32(up, gate, x, N, K, threads=THREADS)
    assert np.linalg.norm(y - yo) / np.linalg.norm(yo) <= 1e-5


def test_workspace_tickets_return_to_zero(cuda):
    N, K = 4096, 4096
    tiles = to_dev(synth.tiles_np(N, K, 81), cuda)
    x = to_dev(synth.x_np(K, 1, 82), cuda)
    for split in (2, 7, 64):
        q4rdna.gemv(tiles, x, split=split)
    torch.cuda.synchronize()
    for ws in q4rdna._WS.values():
        rb = (N + 127) // 128
        assert int(ws[: 4 * rb].view(torch.int32).abs().sum()) == 0


def test_error_statuses_on_device(cuda):
    import ctypes

    N, K = 1024, 4096
    tiles = to_dev(synth.tiles_np(N, K, 91), cuda)
    x = to_dev(synth.x_np(K, 1, 92), cuda)
    y = torch.empty(N, device=cuda)
    L = q4rdna.lib
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert L.q4rdna_gemv(tiles.data_ptr() + 8, x.data_ptr(), y.data_ptr(), N, K, 1, None, None, 0, st) == 3
    assert L.q4rdna_gemv(tiles.data_ptr(), x.data_ptr() + 4, y.data_ptr(), N, K, 1, None, None, 0, st) == 3
    cfg = q4rdna.Cfg()
    cfg.split = 4  # K-ranges added inside a thread-block cluster: no workspace
    assert L.q4rdna_workspace_bytes(N, K, 1, 0, ctypes.byref(cfg)) == 0
    assert L.q4rdna_gemv(tiles.data_ptr(), x.data_ptr(), y.data_ptr(), N, K, 1, ctypes.byref(cfg), None, 0, st) == 0
    cfg.split = 16  # beyond a cluster: partial sums and arrival tickets in the workspace
    need = L.q4rdna_workspace_bytes(N, K, 1, 0, ctypes.byref(cfg))
    assert need > 0
    ws = torch.zeros(need, dtype=torch.uint8, device=cuda)
    assert L.q4rdna_gemv(tiles.data_ptr(), x.data_ptr(), y.data_ptr(), N, K, 1, ctypes.byref(cfg), None, 0, st) == 4
    assert L.q4rdna_gemv(tiles.data_ptr(), x.data_ptr(), y.data_ptr(), N, K, 1, ctypes.byref(cfg),
                         ws.data_ptr(), need - 1, st) == 4
    assert L.q4rdna_gemv(tiles.data_ptr(), x.data_ptr(), y.data_ptr(), N, K, 1, ctypes.byref(cfg),
                         ws.data_ptr(), need, st) == 0
    torch.cuda.synchronize()


def test_plan_matches_oracle_and_is_deterministic(cuda):
    specs = [(4096, 4096, 0), (1024, 4096, 0), (12288, 4096, 2), (4096, 12288, 0), (96, 128, 1), (32, 64, 0)]
    descs, host = [], []
    for i, (N, K, op) in enumerate(specs):
        t = synth.tiles_np(N, K, 500 + i)
        g = synth.tiles_np(N, K, 600 + i) if op == 2 else None
        x = synth.x_np(K, 1, 700 + i)
        a = synth.x_np(N, 1, 800 + i) if op == 1 else None
        d = {"tiles": to_dev(t, cuda), "x": to_dev(x, cuda), "y": torch.empty((1, N), device=cuda), "op": op}
        if op == 2:
            d["gate_tiles"] = to_dev(g, cuda)
        if op == 1:
            d["add"] = to_dev(a, cuda)
        descs.append(d)
        host.append((t, g, x, a))
    plan = q4rdna.Plan(descs, B=1)
    info = plan.info()
    assert info["count"] == len(specs) and info["items"] > 0
    plan.run()
    first = [d["y"].cpu().numpy().copy() for d in descs]
    plan.run()
    for d, f, (N, K, op), (t, g, x, a) in zip(descs, first, specs, host):
        y = d["y"].cpu().numpy()
        assert np.array_equal(y.view(np.uint32), f.view(np.uint32))
        if op == 0:
            y64, mag = oracle.gemv_f64(t, x, N, K, threads=THREADS)
            tolerance.check(y, y64, mag, f"plan {N}x{K}")
        elif op == 1:
            y64, mag = oracle.gemv_f64(t, x, N, K, threads=THREADS)
            tolerance.check(y, y64 + a, mag + np.abs(a), f"plan add {N}x{K}")
        else:
            yo = oracle.gemv_swiglu_f32(t, g, x, N, K, threads=THREADS)
            assert np.linalg.norm(y - yo) / np.linalg.norm(yo) <= 1e-5
    plan.close()


def test_sidecar_and_name_keyed_operators(cuda, tmp_path, monkeypatch):
    """The reference's operator surface: sidecar lookup by ggml name, scope
    filter, shape checks and fallback (source/q4rdna.cu:682-793)."""
    specs = [("blk.0.attn_q.weight", 4096, 4096), ("blk.0.ffn_gate.weight", 1024, 4096),
             ("blk.0.ffn_up.weight", 1024, 4096), ("blk.0.ffn_down.weight", 4096, 1024)]
    tiles = {n: synth.tiles_np(r, c, 900 + i) for i, (n, r, c) in enumerate(specs)}
    path = tmp_path / "model.q4rdna"
    fmt.write_sidecar(str(path), [(n, tiles[n], r, c) for n, r, c in specs])

    sc = q4rdna.Sidecar(str(path), 0)
    assert [e[:3] for e in sc.entries()] == [(n, r, c) for n, r, c in specs]
    rows, cols, ptr = sc.find("blk.0.attn_q.weight")
    assert (rows, cols) == (4096, 4096) and ptr % 256 == 0
    assert sc.find("blk.9.attn_q.weight") is None
    sc.close()

    monkeypatch.setenv("LLAMA_Q4_RDNA_SIDECAR", str(path))
    monkeypatch.delenv("LLAMA_Q4_RDNA_SCOPE", raising=False)
    q4rdna.registry_reset()
    x = synth.x_np(4096, 1, 1)[0]
    xd, yd = to_dev(x, cuda), torch.empty(4096, device=cuda)
    assert q4rdna.mul_mat("blk.0.attn_q.weight", (4096, 4096), xd, yd)
    y64, mag = oracle.gemv_f64(tiles["blk.0.attn_q.weight"], x, 4096, 4096, threads=THREADS)
    tolerance.check(yd.cpu().numpy(), y64, mag, "mul_mat by name")
    assert not q4rdna.mul_mat("blk.0.attn_q.weight", (4096, 1024), xd, yd)   # shape mismatch
    assert not q4rdna.mul_mat("blk.7.attn_q.weight", (4096, 4096), xd, yd)   # unknown name
    add = to_dev(synth.x_np(4096, 1, 2)[0], cuda)
    assert q4rdna.mul_mat_add("blk.0.attn_q.weight", (4096, 4096), xd, add, yd)
    tolerance.check(yd.cpu().numpy(), y64 + add.cpu().numpy(), mag + np.abs(add.cpu().numpy()), "mul_mat_add")
    y2 = torch.empty(1024, device=cuda)
    assert q4rdna.mul_mat_glu("blk.0.ffn_up.weight", (4096, 1024), "blk.0.ffn_gate.weight", (4096, 1024), xd, y2)
    yo = oracle.gemv_swiglu_f32(tiles["blk.0.ffn_up.weight"], tiles["blk.0.ffn_gate.weight"], x, 1024, 4096,
                                threads=THREADS)
    assert np.linalg.norm(y2.cpu().numpy() - yo) / np.linalg.norm(yo) <= 1e-5
    assert q4rdna.registry_hits("blk.0.attn_q.weight") == 2
    assert q4rdna.registry_hits("blk.0.ffn_up.weight") == 1

    monkeypatch.setenv("LLAMA_Q4_RDNA_SCOPE", "ffn")
    assert not q4rdna.mul_mat("blk.0.attn_q.weight", (4096, 4096), xd, yd)   # out of scope
    monkeypatch.setenv("LLAMA_Q4_RDNA_SCOPE", "hotspot")
    assert not q4rdna.mul_mat("blk.0.ffn_down.weight", (1024, 4096), to_dev(synth.x_np(1024, 1, 3)[0], cuda), yd)
    torch.cuda.synchronize()
    q4rdna.registry_reset()


def test_qwen3_8b_decode_step_plan_full_size(cuda):
    """Config 2 at full size (252 tensors, 3.69 GB): deterministic, and spot
    tensors checked against the oracle."""
    names = synth.model_tensors("qwen3-8b")
    descs = []
    for i, (n, N, K) in enumerate(names):
        t = synth.tiles_torch(N, K, synth.BASE_SEED + i, cuda)
        x = torch.randn((1, K), generator=torch.Generator(device=cuda).manual_seed(i), device=cuda)
        descs.append({"tiles": t, "x": x, "y": torch.empty((1, N), device=cuda)})
    plan = q4rdna.Plan(descs, B=1)
    assert plan.info()["weight_bytes"] == 3689938944
    plan.run()
    snap = [d["y"].clone() for d in descs]
    plan.run()
    torch.cuda.synchronize()
    for d, s in zip(descs, snap):
        assert torch.equal(d["y"], s)
    for i in (0, 1, 4, 6, 129, 251):
        n, N, K = names[i]
        t = descs[i]["tiles"].cpu().numpy()
        x = descs[i]["x"].cpu().numpy()
        y64, mag = oracle.gemv_f64(t, x, N, K, threads=THREADS)
        tolerance.check(descs[i]["y"].cpu().numpy(), y64, mag, n)
    plan.close()


def test_shared_workspace_across_shapes(cuda):
    """One workspace reused by calls of growing row counts (the ticket area is
    fixed, so a later call never reads an earlier call's partials as tickets)."""
    import ctypes

    L = q4rdna.lib
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    cfg = q4rdna.Cfg()
    cfg.split = 16  # more K-ranges than a cluster holds: the workspace path
    shapes = [(4096, 12288), (12288, 4096), (1024, 4096), (25600, 5120)]
    need = max(L.q4rdna_workspace_bytes(N, K, 1, 0, ctypes.byref(cfg)) for N, K in shapes)
    assert need > 0
    ws = torch.zeros(need, dtype=torch.uint8, device=cuda)
    for rep in range(2):
        for i, (N, K) in enumerate(shapes):
            tiles = synth.tiles_np(N, K, 300 + i)
            x = synth.x_np(K, 1, 400 + i)
            td, xd = to_dev(tiles, cuda), to_dev(x, cuda)
            y = torch.empty(N, device=cuda)
            assert L.q4rdna_gemv(td.data_ptr(), xd.data_ptr(), y.data_ptr(), N, K, 1, ctypes.byref(cfg),
                                 ws.data_ptr(), need, st) == 0
            y64, mag = oracle.gemv_f64(tiles, x, N, K, threads=THREADS)
            tolerance.check(y.cpu().numpy(), y64, mag, f"shared ws {N}x{K} rep {rep}")
