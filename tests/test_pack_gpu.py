"""GPU sidecar packer (q4rdna_pack_bf16) against the reference packer: byte for
byte on the reference packer's own output (golden file), and against the
oracle's restatement of it (pinned to that file) on typical, adversarial and
random-bit bf16 weights.  Needs a B200."""
import os

import numpy as np
import pytest
import torch

import make_golden
import oracle
import q4rdna
from q4rdna import format as fmt

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
THREADS = max(1, min(16, os.cpu_count() or 1))


def to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """f32 -> bf16 bit patterns, round to nearest even (NaN kept NaN)."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(a)
    r[nan] = 0x7FC0
    return r


def gpu_pack(bits: np.ndarray, cuda) -> np.ndarray:
    w = torch.from_numpy(bits.view(np.int16)).to(cuda)
    return q4rdna.pack_bf16(w).cpu().numpy()


def test_gpu_packer_matches_reference_packer_file(cuda):
    hdr, entries = fmt.read_sidecar(os.path.join(GOLD, "ref_pack_small.q4rdna"))
    data = open(os.path.join(GOLD, "ref_pack_small.q4rdna"), "rb").read()
    inputs = np.load(os.path.join(GOLD, "bf16_inputs.npz"))
    for e in entries:
        bits = inputs[e.name.replace(".", "_")].reshape(e.rows, e.cols)
        assert gpu_pack(bits, cuda).tobytes() == data[e.offset:e.offset + e.size], e.name


def test_gpu_packer_matches_oracle_on_golden_groups(cuda):
    """The 4000 seeded groups pinned against the reference's select_scale (five
    magnitudes from 1e-6 to 300, zero and constant groups), as bf16 rows."""
    bits = to_bf16_bits(make_golden.select_scale_groups())  # 4000 x 64
    assert np.array_equal(gpu_pack(bits, cuda), oracle.pack_bf16(bits, threads=THREADS))


KINDS = ["weights", "tiny", "huge", "sparse", "ties", "random_bits", "specials"]


@pytest.mark.parametrize("kind", KINDS)
def test_gpu_packer_matches_oracle(cuda, kind):
    rng = np.random.default_rng(3000 + KINDS.index(kind))
    N, K = 256, 1024
    if kind == "weights":
        a = rng.standard_normal((N, K)).astype(np.float32) * 0.02
    elif kind == "tiny":  # bf16 subnormals and values whose fp16 scales are subnormal
        a = rng.standard_normal((N, K)).astype(np.float32) * np.exp2(rng.integers(-133, -10, (N, 1)))
    elif kind == "huge":
        a = rng.standard_normal((N, K)).astype(np.float32) * np.exp2(rng.integers(10, 120, (N, 1)))
    elif kind == "sparse":
        a = rng.standard_normal((N, K)).astype(np.float32) * (rng.random((N, K)) < 0.05)
    elif kind == "ties":  # small integers times a power of two: quotients land on half-integers
        a = rng.integers(-17, 18, (N, K)).astype(np.float32) * np.exp2(rng.integers(-12, 4, (N, 1))) / 2
    elif kind == "random_bits":
        bits = rng.integers(0, 1 << 16, (N, K), dtype=np.uint64).astype(np.uint16)
        exp = (bits >> 7) & 0xFF
        bits[exp == 0xFF] &= 0x807F  # finite patterns only here; specials below
        assert np.array_equal(gpu_pack(bits, cuda), oracle.pack_bf16(bits, threads=THREADS))
        return
    else:  # groups holding infinities and NaNs among normal weights
        a = rng.standard_normal((N, K)).astype(np.float32) * 0.02
        a[::7, 3] = np.inf
        a[::11, 70] = -np.inf
        a[::13, 140] = np.nan
    bits = to_bf16_bits(a)
    assert np.array_equal(gpu_pack(bits, cuda), oracle.pack_bf16(bits, threads=THREADS))


def test_pack_sidecar_writes_the_reference_container(cuda, tmp_path):
    """pack_sidecar (GPU packing + the host container writer) reproduces the
    reference packer's whole file."""
    inputs = np.load(os.path.join(GOLD, "bf16_inputs.npz"))
    tensors = []
    for name, rows, cols, _ in make_golden.SMALL:
        bits = inputs[name.replace(".", "_")].reshape(rows, cols)
        tensors.append((name, torch.from_numpy(bits.view(np.int16)).to(cuda)))
    p = tmp_path / "gpu.q4rdna"
    q4rdna.pack_sidecar(str(p), tensors)
    assert p.read_bytes() == open(os.path.join(GOLD, "ref_pack_small.q4rdna"), "rb").read()


def test_pack_argument_errors(cuda):
    import ctypes

    L = q4rdna.lib
    w = torch.zeros((64, 128), dtype=torch.int16, device=cuda)
    t = torch.empty(64 * 128 * 34 // 64, dtype=torch.uint8, device=cuda)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert L.q4rdna_pack_bf16(w.data_ptr(), t.data_ptr(), 48, 128, st) == 2   # rows % 32
    assert L.q4rdna_pack_bf16(w.data_ptr(), t.data_ptr(), 64, 96, st) == 2    # cols % 64
    assert L.q4rdna_pack_bf16(w.data_ptr() + 2, t.data_ptr(), 32, 128, st) == 3
    assert L.q4rdna_pack_bf16(None, t.data_ptr(), 64, 128, st) == 1
    assert L.q4rdna_pack_bf16(w.data_ptr(), t.data_ptr(), 64, 128, st) == 0
    torch.cuda.synchronize()
    assert np.all(t.cpu().numpy() == 0)  # all-zero weights: zero scales, zero codes


def test_pack_cli_reproduces_reference_packer_file(cuda, tmp_path):
    """python -m q4rdna.pack MANIFEST OUTPUT, given the reference packer's own
    manifest format and raw bf16 inputs, writes its file byte for byte."""
    from q4rdna import pack

    inputs = np.load(os.path.join(GOLD, "bf16_inputs.npz"))
    raw = tmp_path / "weights.bin"
    lines, off = [], 16  # a header before the data, as in a safetensors file
    with open(raw, "wb") as f:
        f.write(b"\0" * off)
        for name, rows, cols, _ in make_golden.SMALL:
            b = inputs[name.replace(".", "_")].reshape(rows, cols).astype("<u2")
            f.write(b.tobytes())
            lines.append(f"{raw}\t{off}\t{rows}\t{cols}\t{name}")
            off += b.nbytes
    m = tmp_path / "manifest.tsv"
    m.write_text("\n".join(lines) + "\n")
    out = tmp_path / "out.q4rdna"
    assert pack.main([str(m), str(out)]) == 0
    assert out.read_bytes() == open(os.path.join(GOLD, "ref_pack_small.q4rdna"), "rb").read()
