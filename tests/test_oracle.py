"""The CPU oracle, pinned against the reference's own code and its golden outputs.

No GPU.  The committed fixtures (tests/golden/, made by make_golden.py from the
reference's compiled CPU code and its two packers) pin the oracle wherever the
reference checkout is absent; where oracle/_ref was built the tests also
compare against the reference functions live.
"""
import hashlib
import json
import os

import numpy as np
import pytest

import make_golden
import oracle
from q4rdna import format as fmt, synth

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_oracle_built():
    assert oracle.lib is not None, "make -C oracle"


def test_fp16_to_f32_all_patterns_match_reference_hash():
    meta = json.load(open(os.path.join(GOLD, "ref_fp16.json")))
    tab = np.array([oracle.lib.q4o_fp16_to_f32(h) for h in range(65536)], np.float32)
    assert sha(tab.view(np.uint32)) == meta["fp16_to_f32_all_sha256"]


def test_reference_cpu_decoder_halves_subnormals_ieee_mode_does_not():
    """The reference CPU decoder (q4rdna_cpu_experiment.cpp:53) is IEEE except
    that fp16 subnormals come out at half their value; the IEEE mode equals
    numpy (and the reference GPU kernel's __half2float) on every pattern."""
    h = np.arange(65536, dtype=np.uint16)
    ref = np.array([oracle.lib.q4o_fp16_to_f32(int(v)) for v in h], np.float32)
    ieee = np.array([oracle.lib.q4o_fp16_to_f32_ieee(int(v)) for v in h], np.float32)
    npv = h.view(np.float16).astype(np.float32)
    nan = np.isnan(npv)
    assert np.array_equal(ieee.view(np.uint32)[~nan], npv.view(np.uint32)[~nan]) and np.isnan(ieee[nan]).all()
    sub = ((h & 0x7C00) == 0) & ((h & 0x03FF) != 0)
    assert np.array_equal(ref[sub] * 2, ieee[sub])
    assert np.array_equal(ref.view(np.uint32)[~sub & ~nan], ieee.view(np.uint32)[~sub & ~nan])


def test_f32_to_fp16_matches_reference_hash():
    meta = json.load(open(os.path.join(GOLD, "ref_fp16.json")))
    fl = make_golden.fp16_inputs()
    to16 = np.array([oracle.lib.q4o_f32_to_fp16(float(v)) for v in fl], np.uint16)
    assert sha(to16) == meta["f32_to_fp16_sha256"]


@pytest.mark.skipif(oracle.ref is None, reason="oracle/_ref not built here")
def test_fp16_against_all_three_reference_copies_live():
    for h in range(0, 65536, 7):
        v = oracle.lib.q4o_fp16_to_f32(h)
        for f in (oracle.ref.q4ref_exp_fp16_to_float, oracle.ref.q4ref_pack_fp16_to_float):
            r = f(h)
            assert (np.isnan(v) and np.isnan(r)) or np.float32(v).view(np.uint32) == np.float32(r).view(np.uint32)
        e = (h >> 10) & 31
        if e != 31:  # the bench copy has no inf/nan branch (q4rdna_gemv_bench.hip:163-187)
            r = oracle.ref.q4ref_bench_half_to_float(h)
            assert np.float32(v).view(np.uint32) == np.float32(r).view(np.uint32)


def test_gemv_matches_reference_cpu_gemv_golden():
    """Bit-exact against reference_q4_rdna (q4rdna_gemv_bench.hip:189-211)."""
    g = np.load(os.path.join(GOLD, "ref_bench_gemv.npz"))
    R, C = int(g["rows"]), int(g["cols"])
    tiles = synth.tiles_np(R, C, int(g["seed"]))
    assert sha(tiles) == str(g["tiles_sha256"]), "synthetic generator drifted"
    for xk, yk in (("x_randn", "y_randn"), ("x_sincos", "y_sincos")):
        y = oracle.gemv_f32(tiles, g[xk], R, C, threads=4, decode="refcpu")
        assert np.array_equal(y.view(np.uint32), g[yk].view(np.uint32)), xk


@pytest.mark.skipif(oracle.ref is None, reason="oracle/_ref not built here")
def test_gemv_matches_reference_cpu_gemv_live():
    R, C = oracle.ref.q4ref_bench_rows(), oracle.ref.q4ref_bench_columns()
    tiles = synth.tiles_np(R, C, 99)
    x = synth.x_np(C, 1, 98)[0] * np.float32(1e-3)
    y = oracle.gemv_f32(tiles, x, R, C, threads=4, decode="refcpu")
    yr = oracle.ref_bench_gemv(tiles, x)
    assert np.array_equal(y.view(np.uint32), yr.view(np.uint32))


def test_f64_oracle_close_to_reference_order():
    g = np.load(os.path.join(GOLD, "ref_bench_gemv.npz"))
    R, C = int(g["rows"]), int(g["cols"])
    tiles = synth.tiles_np(R, C, int(g["seed"]))
    y64, mag = oracle.gemv_f64(tiles, g["x_randn"], R, C, threads=4, decode="refcpu")
    nw = np.max(np.abs(g["y_randn"] - y64) / mag)
    assert nw < 2e-6  # the reference's f32 order itself is within ~3e-7 normwise
    # IEEE-decoded y differs from the reference CPU GEMV only through subnormal scales
    y64i, magi = oracle.gemv_f64(tiles, g["x_randn"], R, C, threads=4, decode="ieee")
    assert np.max(np.abs(y64i - y64) / magi) > 1e-4


def test_dequant_matches_format_unpack():
    N, K = 96, 192
    tiles = synth.tiles_np(N, K, 5)
    W = oracle.dequant(tiles, N, K, decode="ieee")
    codes, scales = fmt.unpack_tiles(tiles, N, K)
    ref = codes.astype(np.float32) * np.repeat(scales.astype(np.float32), 64, axis=1)
    assert np.array_equal(W.view(np.uint32), ref.view(np.uint32))


def test_select_scale_matches_reference_packer_golden():
    g = np.load(os.path.join(GOLD, "ref_select_scale.npz"))
    groups = make_golden.select_scale_groups()
    assert sha(groups) == str(g["groups_sha256"])
    ours = np.array([oracle.select_scale(v) for v in groups], np.uint16)
    assert np.array_equal(ours, g["scale_bits"])


def test_packer_matches_reference_cpp_packer_golden():
    hdr, entries = fmt.read_sidecar(os.path.join(GOLD, "ref_pack_small.q4rdna"))
    data = open(os.path.join(GOLD, "ref_pack_small.q4rdna"), "rb").read()
    inputs = np.load(os.path.join(GOLD, "bf16_inputs.npz"))
    assert [(e.name, e.rows, e.cols) for e in entries] == [(n, r, c) for n, r, c, _ in make_golden.SMALL]
    for e in entries:
        tiles = oracle.pack_bf16(inputs[e.name.replace(".", "_")], threads=2)
        assert tiles.tobytes() == data[e.offset:e.offset + e.size], e.name


def test_sidecar_writer_matches_reference_layout_golden(tmp_path):
    """Our writer reproduces the reference packer's whole file byte for byte."""
    hdr, entries = fmt.read_sidecar(os.path.join(GOLD, "ref_pack_small.q4rdna"))
    data = open(os.path.join(GOLD, "ref_pack_small.q4rdna"), "rb").read()
    tensors = [(e.name, np.frombuffer(data[e.offset:e.offset + e.size], np.uint8), e.rows, e.cols) for e in entries]
    p = tmp_path / "ours.q4rdna"
    fmt.write_sidecar(str(p), tensors)
    assert p.read_bytes() == data
    assert hdr["magic"] == fmt.MAGIC and hdr["version"] == 1 and hdr["data_offset"] % 4096 == 0
    assert all(e.offset % 256 == 0 for e in entries)


def test_epilogue_oracles():
    N, K = 64, 128
    up, gate = synth.tiles_np(N, K, 1), synth.tiles_np(N, K, 2)
    x = synth.x_np(K, 2, 3)
    add = synth.x_np(N, 2, 4)
    yu, yg = oracle.gemv_f32(up, x, N, K), oracle.gemv_f32(gate, x, N, K)
    assert not np.array_equal(yu, oracle.gemv_f32(up, x, N, K, decode="refcpu"))
    assert np.array_equal(oracle.gemv_add_f32(up, x, add, N, K), yu + add)
    sw = oracle.gemv_swiglu_f32(up, gate, x, N, K)
    silu = np.array([oracle.lib.q4o_silu(float(v)) for v in yg.reshape(-1)], np.float32).reshape(yg.shape)
    assert np.array_equal(sw, yu * silu)


# ---- Q4_K (the qkv-fallback tensors; q4rdna_cpu_experiment.cpp:102-135) ----

def _q4k_fixture():
    g = np.load(os.path.join(GOLD, "ref_q4k_dequant.npz"))
    return g["blocks"], g["weights"]


def test_q4k_dequant_matches_reference_golden():
    """The oracle's restatement, in the reference CPU decoding, equals the
    reference's dequantize_q4_k bit for bit on the committed blocks (edge blocks
    included: zero, subnormal, negative and maximal d/dmin, 0xFF scale bytes)."""
    blocks, w = _q4k_fixture()
    n = blocks.size // 144
    assert np.array_equal(blocks, make_golden.q4k_blocks())
    W = oracle.q4k_dequant(blocks, n, 256, decode="refcpu").reshape(-1)
    assert np.array_equal(W.view(np.uint32), w.view(np.uint32))


@pytest.mark.skipif(oracle.ref is None, reason="oracle/_ref not built")
def test_q4k_dequant_matches_reference_live():
    blocks = synth.q4k_np(8, 2048, 77)
    W = oracle.q4k_dequant(blocks, 8, 2048, decode="refcpu").reshape(-1)
    assert np.array_equal(W.view(np.uint32), oracle.ref_q4k_dequant(blocks).view(np.uint32))


def test_q4k_ieee_decode_differs_only_through_subnormal_d():
    blocks, _ = _q4k_fixture()
    n = blocks.size // 144
    Wr = oracle.q4k_dequant(blocks, n, 256, decode="refcpu")
    Wi = oracle.q4k_dequant(blocks, n, 256, decode="ieee")
    dd = blocks.reshape(n, 144)[:, :4].copy().view(np.uint16)
    subn = ((dd & 0x7C00) == 0) & ((dd & 0x3FF) != 0)
    same = ~subn.any(axis=1)
    assert np.array_equal(Wr[same].view(np.uint32), Wi[same].view(np.uint32))
    assert not np.array_equal(Wr[~same], Wi[~same])  # the subnormal edge block decodes differently


def test_q4k_gemv_reference_order_close_to_f64():
    N, K, B = 96, 1280, 3
    blocks = synth.q4k_np(N, K, 78)
    x = synth.x_np(K, B, 79)
    y32 = oracle.q4k_gemv_f32(blocks, x, N, K)
    y64, mag = oracle.q4k_gemv_f64(blocks, x, N, K)
    assert np.max(np.abs(y32 - y64) / mag) < 2e-6
    W = oracle.q4k_dequant(blocks, N, K).astype(np.float64)
    assert np.allclose(W @ x.T.astype(np.float64), y64.T, rtol=0, atol=1e-12)
