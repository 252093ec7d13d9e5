"""One rank of the row-sharded (tensor-parallel) CPU check, run by
test_tp_gloo.py as WORLD_SIZE processes over gloo.

Every rank builds the same full tensors and activations, computes only its
row shard of each tensor with the oracle (the checker; the GPU ranks run the
library's plan kernel in its place), packs the slices into its y buffer by
q4rdna.tp.Layout, all-gathers with q4rdna.tp.all_gather and reassembles.  The
assembled outputs must equal the unsharded oracle GEMV bit for bit.
"""

import datetime
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
for p in (REPO, os.path.join(REPO, "rdna-gfx1201-v0.1_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import oracle  # noqa: E402
from q4rdna import synth, tp  # noqa: E402

TENSORS = [("blk.0.attn_q.weight", 256, 512), ("blk.0.attn_k.weight", 128, 1024),
           ("blk.0.ffn_down.weight", 512, 256), ("blk.1.ffn_up.weight", 384, 192)]
B = 2
SEED = 20260816


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    tensors = [(n, N * world // 2, K) for (n, N, K) in TENSORS]  # whole 32-row bands per rank
    lay = tp.Layout(tensors, world, B)
    full, xs = [], []
    y_rank = np.zeros(B * lay.ysz, np.float32)
    for i, (n, N, K) in enumerate(tensors):
        tiles = synth.tiles_np(N, K, SEED + i)
        x = synth.x_np(K, B, SEED + 100 + i)
        full.append(tiles)
        xs.append(x)
        shard = tp.shard_tiles(tiles, N, K, world, rank)
        rows = lay.slots[i].rows
        lay.local_view(y_rank, i)[:] = oracle.gemv_f32(shard, x, rows, K)
    gathered = torch.empty(world * B * lay.ysz, dtype=torch.float32)
    tp.all_gather(torch.from_numpy(y_rank), gathered)
    bad = 0
    for i, (out_np, out_t) in enumerate(zip(lay.assemble(gathered.numpy()), lay.assemble(gathered))):
        n, N, K = tensors[i]
        want = oracle.gemv_f32(full[i], xs[i], N, K)
        if out_np.shape != (B, N) or not np.array_equal(out_np, want):
            print(f"rank {rank}: {n} differs after assembly", flush=True)
            bad += 1
        if not np.array_equal(out_t.numpy(), want):
            print(f"rank {rank}: {n} differs (torch assembly)", flush=True)
            bad += 1
    dist.barrier()
    dist.destroy_process_group()
    return 1 if bad else 0


if __name__ == "__main__":
    sys.exit(main())
