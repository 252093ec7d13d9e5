"""The Q4_K GEMV (q4k_gemv_kernel) and Q4_K dequant against the CPU oracle,
and plans that mix Q4_K and Q4_RDNA tensors (the reference's qkv-fallback
hybrid, source/q4rdna.cu:685-691).  Needs a B200."""
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


def test_q4k_dequant_bit_exact(cuda):
    """Bit-exact with the oracle's IEEE decoding, edge blocks included, and with
    the reference's own dequantiser wherever d and dmin are fp16-normal."""
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "ref_q4k_dequant.npz"))
    blocks, wref = g["blocks"], g["weights"]
    n = blocks.size // 144
    W = q4rdna.q4k_dequant(to_dev(blocks, cuda), n, 256).cpu().numpy()
    Wi = oracle.q4k_dequant(blocks, n, 256, decode="ieee")
    assert np.array_equal(W.view(np.uint32), Wi.view(np.uint32))
    dd = blocks.reshape(n, 144)[:, :4].copy().view(np.uint16)
    normal = ~(((dd & 0x7C00) == 0) & ((dd & 0x3FF) != 0)).any(axis=1)
    assert np.array_equal(W[normal].view(np.uint32), wref.reshape(n, 256)[normal].view(np.uint32))
    N, K = 96, 2304
    b2 = synth.q4k_np(N, K, 5)
    W2 = q4rdna.q4k_dequant(to_dev(b2, cuda), N, K).cpu().numpy()
    assert np.array_equal(W2.view(np.uint32), oracle.q4k_dequant(b2, N, K).view(np.uint32))


@pytest.mark.parametrize("B", [1, 2, 5, 16])
@pytest.mark.parametrize("N,K", [(4096, 4096), (1024, 4096), (200, 768), (4096, 12288), (64, 256), (130, 3072)])
def test_q4k_gemv(cuda, B, N, K):
    blocks = synth.q4k_np(N, K, 100 + N + K + B)
    x = synth.x_np(K, B, 200 + B)
    y = q4rdna.q4k_gemv(to_dev(blocks, cuda), to_dev(x, cuda)).cpu().numpy()
    y64, mag = oracle.q4k_gemv_f64(blocks, x, N, K, threads=THREADS)
    tolerance.check(y, y64, mag, f"q4k B={B} {N}x{K}")


def test_q4k_gemv_add_and_1d(cuda):
    N, K, B = 1024, 4096, 3
    blocks = to_dev(synth.q4k_np(N, K, 300), cuda)
    hb = blocks.cpu().numpy()
    x = synth.x_np(K, B, 301)
    add = synth.x_np(N, B, 302)
    y = q4rdna.q4k_gemv(blocks, to_dev(x, cuda), add=to_dev(add, cuda)).cpu().numpy()
    y64, mag = oracle.q4k_gemv_f64(hb, x, N, K, threads=THREADS)
    tolerance.check(y, y64 + add, mag + np.abs(add), "q4k add")
    y1 = q4rdna.q4k_gemv(blocks, to_dev(x[1], cuda)).cpu().numpy()
    assert y1.shape == (N,)
    yb = q4rdna.q4k_gemv(blocks, to_dev(x, cuda)).cpu().numpy()
    assert np.array_equal(y1.view(np.uint32), yb[1].view(np.uint32)), "a column must not depend on the others"


def test_q4k_gemv_extreme_columns(cuda):
    """Per-sub-block power-of-two scaling of x: zero, tiny, huge and mixed
    columns stay in tolerance; f32-subnormal activations flush to zero."""
    N, K, B = 512, 4096, 8
    blocks = synth.q4k_np(N, K, 400)
    x = synth.x_np(K, B, 401)
    x[1] = 0.0
    x[2] *= 1e-30
    x[3] *= 1e30
    x[4, ::2] *= 1e-6
    x[5, :32] = 0.0
    x[6] = np.float32(1e-40)
    x[7, 100] = 3e4
    y = q4rdna.q4k_gemv(to_dev(blocks, cuda), to_dev(x, cuda)).cpu().numpy()
    y64, mag = oracle.q4k_gemv_f64(blocks, x, N, K, threads=THREADS)
    assert np.all(y[1] == 0.0)
    assert np.all(np.isfinite(y[6])) and np.max(np.abs(y[6])) <= 1e-30
    for b in range(B):
        if b in (1, 6):
            continue
        tolerance.check(y[b], y64[b], mag[b], f"column {b}")


def test_q4k_gemv_deterministic(cuda):
    N, K, B = 4096, 4096, 2
    blocks = to_dev(synth.q4k_np(N, K, 500), cuda)
    x = to_dev(synth.x_np(K, B, 501), cuda)
    a = q4rdna.q4k_gemv(blocks, x).cpu().numpy()
    b = q4rdna.q4k_gemv(blocks, x).cpu().numpy()
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_q4k_errors(cuda):
    blocks = to_dev(synth.q4k_np(64, 512, 1), cuda)
    x = torch.zeros((1, 512), device=cuda)
    y = torch.empty((1, 64), device=cuda)
    L = q4rdna.lib
    assert L.q4rdna_q4k_gemv(blocks.data_ptr(), x.data_ptr(), None, y.data_ptr(), 64, 500, 1, None) == 2  # K % 256
    assert L.q4rdna_q4k_gemv(blocks.data_ptr(), x.data_ptr() + 4, None, y.data_ptr(), 64, 256, 1, None) == 3
    assert L.q4rdna_q4k_gemv(blocks.data_ptr(), x.data_ptr(), None, y.data_ptr(), 64, 512, 17, None) == 5
    assert L.q4rdna_q4k_gemv(None, x.data_ptr(), None, y.data_ptr(), 64, 512, 1, None) == 1
    assert L.q4rdna_q4k_bytes(64, 512) == 64 * 2 * 144 and L.q4rdna_q4k_bytes(64, 500) == 0
    d = {"tiles": blocks, "x": x, "y": y, "format": q4rdna.FORMAT_Q4K, "op": q4rdna.OP_SWIGLU, "gate_tiles": blocks}
    with pytest.raises(q4rdna.Q4RDNAError):
        q4rdna.Plan([d], B=1)


def _hybrid_descs(cuda, B, layers=2):
    """A Qwen3-8B-shaped qkv-fallback hybrid: attn_q/k/v in Q4_K, the rest in
    Q4_RDNA (one SwiGLU pair and one add per layer)."""
    descs, host = [], []
    for L in range(layers):
        for i, (name, N, K) in enumerate(synth.QWEN3_8B_LAYER):
            if name == "ffn_up.weight":
                continue
            seed = 9000 + 10 * L + i
            x = synth.x_np(K, B, seed + 500)
            d = {"x": to_dev(x, cuda), "y": torch.empty((B, N), device=cuda)}
            if name.startswith("attn_q") or name.startswith("attn_k") or name.startswith("attn_v"):
                w = synth.q4k_np(N, K, seed)
                d.update(tiles=to_dev(w, cuda), format=q4rdna.FORMAT_Q4K)
                host.append(("q4k", w, None, x, None))
            else:
                w = synth.tiles_np(N, K, seed)
                d["tiles"] = to_dev(w, cuda)
                g = a = None
                if name == "ffn_gate.weight":
                    g = synth.tiles_np(N, K, seed + 1)
                    d.update(op=q4rdna.OP_SWIGLU, gate_tiles=to_dev(g, cuda))
                if name == "attn_output.weight":
                    a = synth.x_np(N, B, seed + 600)
                    d.update(op=q4rdna.OP_ADD, add=to_dev(a, cuda))
                host.append(("q4rdna", w, g, x, a))
            descs.append(d)
    return descs, host


@pytest.mark.parametrize("B", [1, 4])
def test_hybrid_plan_matches_oracle_and_single_calls(cuda, B):
    descs, host = _hybrid_descs(cuda, B)
    plan = q4rdna.Plan(descs, B=B)
    info = plan.info()
    assert info["count"] == len(descs)
    plan.run()
    first = [d["y"].cpu().numpy().copy() for d in descs]
    plan.run()
    for d, f, (kind, w, g, x, a) in zip(descs, first, host):
        y = d["y"].cpu().numpy()
        assert np.array_equal(y.view(np.uint32), f.view(np.uint32)), "plan runs differ"
        N, K = y.shape[1], x.shape[1]
        if kind == "q4k":
            y64, mag = oracle.q4k_gemv_f64(w, x, N, K, threads=THREADS)
            tolerance.check(y, y64, mag, f"hybrid q4k {N}x{K}")
            single = q4rdna.q4k_gemv(d["tiles"], d["x"]).cpu().numpy()
            assert np.array_equal(single.view(np.uint32), y.view(np.uint32)), "plan and single call differ"
        else:
            y64, mag = oracle.gemv_f64(w, x, N, K, threads=THREADS)
            if g is not None:
                g64, mg = oracle.gemv_f64(g, x, N, K, threads=THREADS)
                silu = g64 / (1.0 + np.exp(-g64))
                tolerance.check(y, y64 * silu, mag * np.abs(silu) + np.abs(y64) * 1.1 * mg, "hybrid swiglu")
            elif a is not None:
                tolerance.check(y, y64 + a, mag + np.abs(a), "hybrid add")
            else:
                tolerance.check(y, y64, mag, f"hybrid q4rdna {N}x{K}")
    plan.close()
    assert q4rdna.take_fault() == 0


def test_q4k_only_plan_and_run_host(cuda):
    """A plan of Q4_K tensors alone; run_host on a hybrid plan equals copy-in,
    run, copy-out."""
    B = 2
    K = 4096
    x_dev = torch.empty(B * K, dtype=torch.float32, device=cuda)
    shapes = [4096, 1024, 1024]
    y_dev = torch.empty(B * sum(shapes), dtype=torch.float32, device=cuda)
    descs, off = [], 0
    for i, N in enumerate(shapes):
        descs.append({"tiles": to_dev(synth.q4k_np(N, K, 700 + i), cuda), "x": x_dev.view(B, K),
                      "y": y_dev[off:off + B * N].view(B, N), "format": q4rdna.FORMAT_Q4K})
        off += B * N
    plan = q4rdna.Plan(descs, B=B)
    x_host = torch.from_numpy(synth.x_np(K, B, 710).reshape(-1)).pin_memory()
    y_host = torch.empty(B * sum(shapes), dtype=torch.float32).pin_memory()
    x_dev.copy_(x_host)
    plan.run()
    want = y_dev.cpu().numpy().view(np.uint32).copy()
    x_dev.zero_()
    plan.run_host(x_host, x_dev, y_dev, y_host)
    torch.cuda.current_stream().synchronize()
    assert np.array_equal(y_host.numpy().view(np.uint32), want)
    plan.close()


def _host_step(cuda, B, shared_x, seed):
    """Two Qwen3-8B-shaped layers of the qkv-fallback hybrid with every input
    and output in one device buffer each (run_host's contract).  The Q4_K
    tensors (q, k, v, reading one x per layer) come first in both buffers;
    with shared_x the Q4_RDNA attn_output reads layer 0's q/k/v input too, so
    the Q4_K ranges meet a Q4_RDNA segment's."""
    layers = [[(n, N, K) for (n, N, K) in synth.QWEN3_8B_LAYER] for _ in range(2)]
    qkv = [(L, t) for L in range(2) for t in layers[L] if t[0].split(".")[0] in ("attn_q", "attn_k", "attn_v")]
    rest = [(L, t) for L in range(2) for t in layers[L] if t[0].split(".")[0] not in ("attn_q", "attn_k", "attn_v")]
    xs, ys = {}, {}
    xo = yo = 0
    for L, (name, N, K) in qkv + rest:
        key = ("qkv", L) if (L, name) in [(a, b[0]) for a, b in qkv] else (L, name)
        if key not in xs:
            xs[key] = xo
            xo += B * K
        ys[(L, name)] = yo
        yo += B * N
    x_dev = torch.empty(xo, dtype=torch.float32, device=cuda)
    y_dev = torch.empty(yo, dtype=torch.float32, device=cuda)
    descs = []
    for i, (L, (name, N, K)) in enumerate(qkv + rest):
        seed_i = seed + 10 * L + i
        is_q4k = (L, name) in [(a, b[0]) for a, b in qkv]
        key = ("qkv", L) if is_q4k else (L, name)
        if shared_x and name == "attn_output.weight" and L == 0:
            key = ("qkv", 0)
        xoff = xs[key]
        d = {"x": x_dev[xoff:xoff + B * K].view(B, K), "y": y_dev[ys[(L, name)]:ys[(L, name)] + B * N].view(B, N)}
        if is_q4k:
            d.update(tiles=to_dev(synth.q4k_np(N, K, seed_i), cuda), format=q4rdna.FORMAT_Q4K)
        else:
            d["tiles"] = to_dev(synth.tiles_np(N, K, seed_i), cuda)
            if name == "ffn_gate.weight":
                d.update(op=q4rdna.OP_SWIGLU, gate_tiles=to_dev(synth.tiles_np(N, K, seed_i + 1), cuda))
        descs.append(d)
    x_host = torch.from_numpy(np.random.default_rng(seed).standard_normal(xo, dtype=np.float32)).pin_memory()
    return q4rdna.Plan(descs, B=B), x_dev, y_dev, x_host, yo


@pytest.mark.parametrize("B", [1, 4])
@pytest.mark.parametrize("shared_x", [False, True])
def test_hybrid_run_host_equals_copies_and_run(cuda, B, shared_x):
    """run_host on a plan mixing Q4_K and Q4_RDNA tensors: the Q4_K launch and
    its copies run as one more segment beside the Q4_RDNA segments (or, when
    their byte ranges meet, the whole plan is copied in, run and copied out).
    Either way the outputs are exactly those of copy-in, run, copy-out, into a
    pinned (mapped) or a pageable output buffer, call after call."""
    plan, x_dev, y_dev, x_host, ny = _host_step(cuda, B, shared_x, 9400 + B)
    x_dev.copy_(x_host)
    plan.run()
    want = y_dev.cpu().numpy().view(np.uint32).copy()
    for y_host in (torch.empty(ny, dtype=torch.float32).pin_memory(), torch.empty(ny, dtype=torch.float32)):
        for segments in (0, 3):
            for rep in range(2):
                x_dev.zero_()
                y_dev.fill_(float("nan"))
                y_host.fill_(float("nan"))
                plan.run_host(x_host, x_dev, y_dev, y_host, segments=segments)
                torch.cuda.current_stream().synchronize()
                assert np.array_equal(y_host.numpy().view(np.uint32), want), (segments, rep)
    plan.close()
    assert q4rdna.take_fault() == 0
