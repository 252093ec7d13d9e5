"""Row-sharded tensor parallelism on the CPU: shard arithmetic, layout and the
gather/assemble path, with world_size 2 and 4 gloo ranks (tests/tp_worker.py)."""

import os
import socket
import subprocess
import sys

import numpy as np
import pytest

from q4rdna import synth, tp

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run_ranks(world: int):
    port = _free_port()
    procs = []
    for r in range(world):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE=str(world), LOCAL_RANK=str(r),
                   MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), CUDA_VISIBLE_DEVICES="")
        procs.append(subprocess.Popen([sys.executable, os.path.join(HERE, "tp_worker.py")], env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True))
    outs = []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=180)
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
        outs.append((p.returncode, out))
    return outs


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_equals_unsharded(world):
    outs = _run_ranks(world)
    for r, (rc, out) in enumerate(outs):
        assert rc == 0, f"rank {r} exit {rc}:\n{out}"


def test_shard_rows_and_tiles():
    N, K = 256, 192
    t = synth.tiles_np(N, K, 7)
    band = (K // 64) * 1088
    parts = [tp.shard_tiles(t, N, K, 4, r) for r in range(4)]
    assert [tp.shard_rows(N, 4, r) for r in range(4)] == [(0, 64), (64, 64), (128, 64), (192, 64)]
    assert all(p.shape[0] == 2 * band for p in parts)
    assert np.array_equal(np.concatenate(parts), t)  # the shards tile the stream exactly
    assert np.shares_memory(parts[1], t)             # slices, not copies


@pytest.mark.parametrize("N,world", [(96, 2), (32, 2), (256, 3)])
def test_shard_rejects_partial_bands(N, world):
    with pytest.raises(ValueError):
        tp.shard_rows(N, world, 0)


def test_shard_rejects_wrong_stream_size():
    t = synth.tiles_np(64, 128, 1)
    with pytest.raises(ValueError):
        tp.shard_tiles(t[:-1], 64, 128, 2, 0)
    with pytest.raises(ValueError):
        tp.shard_rows(64, 2, 2)


def test_layout_offsets_and_assemble():
    tensors = [("a", 128, 64), ("b", 64, 128)]
    lay = tp.Layout(tensors, world=2, B=2)
    assert lay.ysz == 64 + 32 and lay.xsz == 192
    assert [(s.rows, s.offset) for s in lay.slots] == [(64, 0), (32, 64)]
    # rank r writes value 1000*r + 100*b + local row into tensor slices
    g = np.zeros((2, 2 * lay.ysz), np.float32)
    for r in range(2):
        for i, s in enumerate(lay.slots):
            v = lay.local_view(g[r], i)
            v[:] = 1000 * r + 100 * np.arange(2)[:, None] + np.arange(s.rows)[None, :]
    a, b = lay.assemble(g.reshape(-1))
    assert a.shape == (2, 128) and b.shape == (2, 64)
    assert a[1, 70] == 1000 * 1 + 100 * 1 + 6 and a[0, 5] == 5
    assert b[0, 31] == 31 and b[1, 32] == 1000 + 100
    # tensor-major blocks: tensor b's batch row 1 of rank 0 starts at float 2*64 + 32
    assert g[0, 2 * 64 + 32] == 100
