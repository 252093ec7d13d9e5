"""Host-side format, C-ABI exports and sidecar validation.  No GPU needed."""
import os
import re
import struct

import numpy as np
import pytest

import q4rdna
from q4rdna import format as fmt, synth

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER_H = os.path.join(REPO, "include", "q4rdna.h")


def declared_symbols():
    src = re.sub(r"/\*.*?\*/", "", open(HEADER_H).read(), flags=re.S)
    return sorted(set(re.findall(r"\b(q4rdna_[a-z_0-9]+)\s*\(", src)))


def test_library_loads_and_exports_every_declared_symbol():
    assert q4rdna.lib is not None, "libq4rdna.so not built"
    decl = declared_symbols()
    assert len(decl) >= 25
    for name in decl:
        assert hasattr(q4rdna.lib, name), name
    assert sorted(q4rdna.SYMBOLS) == decl


def test_status_strings_and_version():
    assert q4rdna.status_string(0) == "ok"
    assert "workspace" in q4rdna.status_string(4)
    assert "sm_100a" in q4rdna.version()


def test_tile_layout_known_answer():
    """Hand-built tile: row r, column k carries code ((r + k) % 16) - 8."""
    N, K = 32, 64
    codes = np.array([[((r + k) % 16) - 8 for k in range(K)] for r in range(N)], np.int8)
    scales = np.arange(1, N + 1, dtype=np.float16).reshape(N, 1)
    t = fmt.pack_tiles(codes, scales)
    assert t.size == 1088
    assert struct.unpack_from("<e", t, 2 * 5)[0] == 6.0                       # scale of row 5
    r, i = 7, 3                                                              # byte 64 + 32 i + r
    b = int(t[64 + 32 * i + r])
    assert (b & 15) == (codes[r, 2 * i] & 15) and (b >> 4) == (codes[r, 2 * i + 1] & 15)
    c2, s2 = fmt.unpack_tiles(t, N, K)
    assert np.array_equal(c2, codes) and np.array_equal(s2, scales)


def test_pack_unpack_round_trip_multi_tile():
    N, K = 160, 320
    rng = np.random.default_rng(0)
    codes = rng.integers(-8, 8, (N, K)).astype(np.int8)
    scales = (np.abs(rng.standard_normal((N, K // 64))) * 0.003).astype(np.float16)
    t = fmt.pack_tiles(codes, scales)
    assert t.size == fmt.tensor_bytes(N, K)
    c2, s2 = fmt.unpack_tiles(t, N, K)
    assert np.array_equal(c2, codes) and np.array_equal(s2.view(np.uint16), scales.view(np.uint16))


def test_synth_distributions():
    t = synth.tiles_np(1024, 4096, 1)
    codes, scales = fmt.unpack_tiles(t, 1024, 4096)
    assert codes.min() == -8 and codes.max() == 7
    hist = np.bincount((codes.astype(np.int16) + 8).reshape(-1), minlength=16) / codes.size
    assert np.all(np.abs(hist - 1 / 16) < 2e-3)
    s = scales.astype(np.float64)
    assert abs(s.mean() - 0.003 * np.sqrt(2 / np.pi)) < 2e-5
    sub = np.mean(np.abs(scales.view(np.uint16) & 0x7C00) == 0)
    assert 0.01 < sub < 0.025  # ~1.6% of scales are fp16 subnormals


def write_valid(tmp_path, name="s.q4rdna"):
    p = tmp_path / name
    fmt.write_sidecar(str(p), [("blk.0.attn_q.weight", synth.tiles_np(64, 128, 1), 64, 128),
                               ("blk.0.ffn_up.weight", synth.tiles_np(32, 64, 2), 32, 64)])
    return p


def open_status(path):
    import ctypes

    h = ctypes.c_void_p()
    st = q4rdna.lib.q4rdna_sidecar_open(str(path).encode(), 0, ctypes.byref(h))
    if st == 0:
        q4rdna.lib.q4rdna_sidecar_close(h)
    return st


def mutate(p, off, fmtc, value):
    b = bytearray(p.read_bytes())
    struct.pack_into(fmtc, b, off, value)
    p.write_bytes(bytes(b))


@pytest.mark.parametrize("case,expect", [
    ("bad_magic", 8), ("bad_version", 8), ("bad_group", 8), ("bad_tile_bytes", 8),
    ("entry_before_data", 8), ("entry_past_end", 8), ("size_mismatch", 8), ("rows_not_32", 8),
    ("cols_not_64", 8), ("name_unterminated", 8), ("misaligned_entry", 8),
    ("truncated_index", 7), ("truncated_data", 7), ("missing_file", 7),
])
def test_sidecar_validation_rejects(tmp_path, case, expect):
    """Rules of source/q4rdna.cu:131-152 (plus 16-byte tensor alignment)."""
    p = write_valid(tmp_path)
    H, E = fmt.HEADER.size, fmt.ENTRY.size
    if case == "bad_magic":
        mutate(p, 0, "<8s", b"Q4RDNA2\x00")
    elif case == "bad_version":
        mutate(p, 8, "<I", 2)
    elif case == "bad_group":
        mutate(p, 16, "<I", 32)
    elif case == "bad_tile_bytes":
        mutate(p, 24, "<I", 1024)
    elif case == "entry_before_data":
        mutate(p, H + 72, "<Q", 64)
    elif case == "entry_past_end":
        mutate(p, H + 72, "<Q", 1 << 40)
    elif case == "size_mismatch":
        mutate(p, H + 80, "<Q", 4351)
    elif case == "rows_not_32":
        mutate(p, H + 64, "<I", 48)
    elif case == "cols_not_64":
        mutate(p, H + 68, "<I", 96)
    elif case == "name_unterminated":
        mutate(p, H, "<64s", b"x" * 64)
    elif case == "misaligned_entry":
        hdr, es = fmt.read_sidecar(str(p))
        mutate(p, H + E + 72, "<Q", es[1].offset - 8)
    elif case == "truncated_index":
        p.write_bytes(p.read_bytes()[:H + E + 10])
    elif case == "truncated_data":
        p.write_bytes(p.read_bytes()[:-100])
    elif case == "missing_file":
        p = tmp_path / "nope.q4rdna"
    assert open_status(p) == expect


def test_name_ops_fall_back_without_sidecar(monkeypatch):
    """LLAMA_Q4_RDNA_SIDECAR unset => return false, no CUDA touched (q4rdna.cu:718-726)."""
    monkeypatch.delenv("LLAMA_Q4_RDNA_SIDECAR", raising=False)
    q4rdna.registry_reset()
    L = q4rdna.lib
    assert L.q4rdna_mul_mat(b"blk.0.attn_q.weight", 4096, 4096, 8, 4096, 8, 4096, None) == 0
    assert L.q4rdna_mul_mat_add(b"blk.0.attn_q.weight", 4096, 4096, 8, 4096, 8, 4096, 8, 4096, None) == 0
    assert L.q4rdna_mul_mat_glu(b"a", 1, 1, b"b", 1, 1, 8, 1, 8, 1, None) == 0
    assert L.q4rdna_mul_mat(b"blk.0.attn_q.weight", 4096, 4096, None, 4096, None, 4096, None) == 0


def test_argument_errors_without_gpu():
    L = q4rdna.lib
    assert L.q4rdna_gemv(8, 8, 8, 4080, 4096, 1, None, None, 0, None) == 2       # N % 32
    assert L.q4rdna_gemv(8, 8, 8, 4096, 4000, 1, None, None, 0, None) == 2       # K % 64
    assert L.q4rdna_gemv(8, 8, 8, 4096, 4096, 0, None, None, 0, None) == 5       # B
    assert L.q4rdna_gemv(8, 8, 8, 4096, 4096, 17, None, None, 0, None) == 5
    assert L.q4rdna_gemv(None, 8, 8, 4096, 4096, 1, None, None, 0, None) == 1
    assert L.q4rdna_gemv_add(16, 8, None, 8, 4096, 4096, 1, None, None, 0, None) == 1
    assert L.q4rdna_gemv_swiglu(16, None, 8, 8, 4096, 4096, 1, None, None, 0, None) == 1
    assert L.q4rdna_plan_create(None, 0, 1, None) == 1
