"""Manifest parsing of the GPU packer's command line (q4rdna.pack), with the
reference packer's rules (source/q4rdna_sidecar_pack.cpp:182-203).  CPU only."""
import numpy as np
import pytest

from q4rdna import pack


def _write(tmp_path, text):
    p = tmp_path / "m.tsv"
    p.write_text(text)
    return str(p)


def test_manifest_lines(tmp_path):
    m = _write(tmp_path, "a.bin\t0\t32\t64\tblk.0.attn_q.weight\n\nb.bin\t128\t64\t128\tname with spaces\n")
    e = pack.read_manifest(m)
    assert [(x.path, x.offset, x.rows, x.cols, x.name) for x in e] == [
        ("a.bin", 0, 32, 64, "blk.0.attn_q.weight"), ("b.bin", 128, 64, 128, "name with spaces")]


@pytest.mark.parametrize("line", ["a.bin\t0\t32\t64", "a.bin\tx\t32\t64\tn", "a.bin\t0\t32\n", "\t0\t32\t64\tn"])
def test_manifest_rejects_malformed_lines(tmp_path, line):
    with pytest.raises(ValueError, match="invalid manifest line"):
        pack.read_manifest(_write(tmp_path, line + "\n"))


@pytest.mark.parametrize("line", ["a.bin\t0\t48\t64\tn", "a.bin\t0\t32\t96\tn", "a.bin\t0\t32\t64\t" + "x" * 64])
def test_manifest_rejects_unsupported_tensors(tmp_path, line):
    with pytest.raises(ValueError, match="unsupported tensor"):
        pack.read_manifest(_write(tmp_path, line + "\n"))


def test_read_bf16_at_offset(tmp_path):
    raw = np.arange(100 + 32 * 64, dtype="<u2")
    f = tmp_path / "w.bin"
    raw.tofile(f)
    e = pack.ManifestEntry(str(f), 200, 32, 64, "t")
    assert np.array_equal(pack.read_bf16(e), raw[100:].reshape(32, 64))
    with pytest.raises(ValueError, match="failed to read"):
        pack.read_bf16(pack.ManifestEntry(str(f), 400, 32, 64, "t"))


def test_cli_usage():
    assert pack.main([]) == 2
