#!/usr/bin/env python3
"""Regenerate the golden fixtures in tests/golden/ from the reference's own code.

Runs only where the reference checkout and oracle/_ref (built by
`make -C oracle`) exist.  Every fixture is produced by the reference itself:

* ref_pack_small.q4rdna: three seeded BF16 matrices packed by the reference
  C++ packer (source/q4rdna_sidecar_pack.cpp, built unmodified into
  oracle/_ref/q4rdna_sidecar_pack).  The same matrices are also packed by the
  reference Python packer (source/pack_q4rdna_sidecar.py: quantize and
  pack_tensor, imported); the script asserts both give identical tile bytes,
  except the sign of a zero scale (all-zero group: Python -0.0, C++ +0.0).
  bf16_inputs.npz holds the BF16 inputs.
* ref_bench_gemv.npz: y of the reference CPU GEMV (reference_q4_rdna,
  source/q4rdna_gemv_bench.hip:189-211, compiled from the file) at its fixed
  12288 x 4096 shape on tiles from q4rdna.synth.tiles_np, for two activations:
  N(0,1) and the bench's own sin/cos vector (q4rdna_gemv_bench.hip:224-227).
  Tiles are regenerated from the seed; their sha256 is stored.
* ref_select_scale.npz: the reference packer's select_scale
  (q4rdna_sidecar_pack.cpp:140-179) on 4000 seeded groups of mixed scale.
* ref_fp16.json: sha256 of the reference fp16->f32 table over all 65536
  patterns (q4rdna_cpu_experiment.cpp:39-60) and of f32->fp16 on 2^20 seeded
  floats plus edge cases (q4rdna_cpu_experiment.cpp:62-100).
* ref_q4k_dequant.npz: the reference's Q4_K block dequantiser
  (dequantize_q4_k, q4rdna_cpu_experiment.cpp:112-135, compiled from the file)
  on Q4_K blocks from q4rdna.synth.q4k_np plus edge blocks (q4k_blocks()):
  the blocks and their 256 f32 weights each.

`python make_golden.py` writes all of them; `--only q4k` only the last.
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "rdna-gfx1201-v0.1_b200"))
# The reference checkout: $Q4RDNA_REFERENCE, else the directory "reference"
# beside this repository.
REF_SRC = os.path.join(os.environ.get("Q4RDNA_REFERENCE") or os.path.join(os.path.dirname(REPO), "reference"),
                       "source")

import oracle  # noqa: E402
from q4rdna import format as fmt, synth  # noqa: E402

SMALL = [("blk.0.attn_k.weight", 64, 128, 101), ("blk.0.ffn_up.weight", 96, 256, 102),
         ("blk.1.attn_q.weight", 32, 64, 103)]
GEMV_SEED = 20260816
X_SEED = 20260817


def bf16_matrix(rows, cols, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    w[0, :64] = 0.0                       # an all-zero group (scale 0)
    w[1, :64] = 0.0125                    # a constant group
    w[2, 64 % cols:64 % cols + 64] *= 100 # a wide group
    bits = w.view(np.uint32)
    return ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16).astype(np.uint16)  # RNE to bf16


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def ref_python_packer():
    spec = importlib.util.spec_from_file_location("ref_pack_py", os.path.join(REF_SRC, "pack_q4rdna_sidecar.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def q4k_blocks() -> np.ndarray:
    """64 seeded Q4_K blocks (4 rows x 4096 columns) and 8 edge blocks: zero
    d and dmin, fp16-subnormal d and dmin, all scale/min bytes 0xFF, negative
    d, d = dmin = 65504, all quant bytes 0x00 / 0xFF."""
    b = synth.q4k_np(4, 4096, 31).reshape(-1, 144).copy()
    e = synth.q4k_np(1, 8 * 256, 32).reshape(-1, 144).copy()
    h = lambda v: np.array([v], np.float16).view(np.uint8)  # noqa: E731
    e[0, :4] = 0
    e[1, 0:2], e[1, 2:4] = h(3e-6), h(1e-7)
    e[2, 4:16] = 0xFF
    e[3, 0:2] = h(-0.002)
    e[4, 0:2], e[4, 2:4] = h(65504.0), h(65504.0)
    e[5, 16:] = 0x00
    e[6, 16:] = 0xFF
    e[7, 4:16] = np.arange(12, dtype=np.uint8) * 21
    return np.concatenate([b, e]).reshape(-1)


def write_q4k():
    blocks = q4k_blocks()
    w = oracle.ref_q4k_dequant(blocks)
    np.savez_compressed(os.path.join(HERE, "ref_q4k_dequant.npz"), blocks=blocks, weights=w)


def main():
    assert oracle.ref is not None and os.path.exists(oracle.REF_PACK_BIN), "build oracle/_ref first"
    if sys.argv[1:] == ["--only", "q4k"]:
        write_q4k()
        print("ref_q4k_dequant.npz written to", HERE)
        return
    # 1. packers
    mats = {name: bf16_matrix(r, c, s) for name, r, c, s in SMALL}
    np.savez_compressed(os.path.join(HERE, "bf16_inputs.npz"), **{n.replace(".", "_"): m for n, m in mats.items()})
    with tempfile.TemporaryDirectory() as td:
        manifest = os.path.join(td, "manifest.tsv")
        with open(manifest, "w") as f:
            for name, r, c, _ in SMALL:
                p = os.path.join(td, name + ".bf16")
                mats[name].tofile(p)
                f.write(f"{p}\t0\t{r}\t{c}\t{name}\n")
        out = os.path.join(HERE, "ref_pack_small.q4rdna")
        subprocess.run([oracle.REF_PACK_BIN, manifest, out], check=True, capture_output=True,
                       env=dict(os.environ, OMP_NUM_THREADS="1"))
    import torch

    py = ref_python_packer()
    packer_notes = []
    hdr, entries = fmt.read_sidecar(out)
    data = open(out, "rb").read()
    for e, (name, r, c, _) in zip(entries, SMALL):
        w = torch.from_numpy(mats[name].astype(np.int16)).view(torch.bfloat16)
        import io

        buf = io.BytesIO()
        py.pack_tensor(buf, w, 4)
        a = np.frombuffer(buf.getvalue(), np.uint8)
        b = np.frombuffer(data[e.offset:e.offset + e.size], np.uint8)
        # The one known difference: for an all-zero group the Python packer stores
        # scale -0.0 (0x8000) where the C++ packer stores +0.0.  Dequantised
        # values are zero either way.  Everything else must be byte-identical.
        diff = np.nonzero(a != b)[0]
        sa = fmt.unpack_tiles(a, r, c)[1].view(np.uint16)
        sb = fmt.unpack_tiles(b, r, c)[1].view(np.uint16)
        signed_zero = (sa != sb) & ((sa | sb) == 0x8000)
        assert ((sa == sb) | signed_zero).all(), f"C++ and Python packers differ in scales of {name}"
        tile_off = diff % fmt.TILE_BYTES
        assert ((tile_off < 64) & (tile_off % 2 == 1)).all(), f"C++ and Python packers differ in codes of {name}"
        packer_notes.append({"tensor": name, "differing_bytes": int(diff.size),
                             "zero_scale_sign_differences": int(signed_zero.sum())})
    # 2. reference CPU GEMV at 12288 x 4096
    R, C = oracle.ref.q4ref_bench_rows(), oracle.ref.q4ref_bench_columns()
    tiles = synth.tiles_np(R, C, GEMV_SEED)
    x0 = synth.x_np(C, 1, X_SEED)[0]
    i = np.arange(C, dtype=np.float32)
    x1 = (np.sin(i * np.float32(0.013)) * np.float32(0.25) + np.cos(i * np.float32(0.007)) * np.float32(0.125)).astype(np.float32)
    y0 = oracle.ref_bench_gemv(tiles, x0)
    y1 = oracle.ref_bench_gemv(tiles, x1)
    np.savez_compressed(os.path.join(HERE, "ref_bench_gemv.npz"), rows=R, cols=C, seed=GEMV_SEED, x_seed=X_SEED,
                        tiles_sha256=sha(tiles), x_randn=x0, x_sincos=x1, y_randn=y0, y_sincos=y1)
    # 3. select_scale
    groups = select_scale_groups()
    ss = np.array([oracle.ref.q4ref_pack_select_scale(g.ctypes.data_as(oracle._f32p)) for g in groups], np.uint16)
    np.savez_compressed(os.path.join(HERE, "ref_select_scale.npz"), groups_sha256=sha(groups), scale_bits=ss)
    # 4. fp16 conversions
    tab = np.array([oracle.ref.q4ref_exp_fp16_to_float(h) for h in range(65536)], np.float32)
    fl = fp16_inputs()
    to16 = np.array([oracle.ref.q4ref_exp_float_to_fp16(float(v)) for v in fl], np.uint16)
    json.dump({"fp16_to_f32_all_sha256": sha(tab.view(np.uint32)),
               "f32_to_fp16_inputs": "tests/golden/make_golden.py:fp16_inputs()",
               "f32_to_fp16_sha256": sha(to16),
               "packer_cpp_vs_python": packer_notes}, open(os.path.join(HERE, "ref_fp16.json"), "w"), indent=1)
    # 5. Q4_K dequantiser
    write_q4k()
    print("golden fixtures written to", HERE)


def select_scale_groups() -> np.ndarray:
    """4000 seeded 64-weight groups at five magnitudes, plus edge groups."""
    rng = np.random.default_rng(7)
    groups = (rng.standard_normal((4000, 64)) * rng.choice([1e-6, 1e-3, 0.02, 1.0, 300.0], (4000, 1))).astype(np.float32)
    groups[:5] = 0.0
    groups[5] = 1.0
    groups[6] = -1.0
    groups[7, :] = 0.0
    groups[7, 3] = 2.5
    return groups


def fp16_inputs() -> np.ndarray:
    """2^20 seeded f32 values spanning fp16 normal, subnormal, overflow, ties."""
    rng = np.random.default_rng(11)
    a = (rng.standard_normal(1 << 19) * np.exp2(rng.integers(-30, 20, 1 << 19))).astype(np.float32)
    b = rng.integers(0, 1 << 32, 1 << 19, dtype=np.uint64).astype(np.uint32).view(np.float32)
    b = b[np.isfinite(b)]
    edge = np.array([0.0, -0.0, 65504.0, 65520.0, 65519.99, 6.1035156e-05, 5.9604645e-08, 2.9802322e-08,
                     2.9802326e-08, 1.0009766, 1.0004883, -1.0004883], np.float32)
    return np.concatenate([edge, a, b]).astype(np.float32)


if __name__ == "__main__":
    main()
