"""One GPU rank of the row-sharded (tensor-parallel) parity check, launched by
test_tp_gpu.py under torch.distributed.run with one process per GPU (NCCL).

Every rank holds the same full tensors on the host, uploads only its row shard
of each (q4rdna.tp.shard_tiles), runs all shards as one plan launch, gathers
the y slices with one NCCL all-gather and reassembles them.  The assembled
outputs must be within tolerance of the unsharded fp64 oracle, and equal bit
for bit to a single-GPU plan over the same shards (rows are independent).
"""

import datetime
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
for p in (HERE, REPO, os.path.join(REPO, "rdna-gfx1201-v0.1_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import oracle  # noqa: E402
import q4rdna  # noqa: E402
import tolerance  # noqa: E402
from q4rdna import synth, tp  # noqa: E402

# Qwen3-8B q / k / down / gate shapes, plus one small ragged-K tensor
TENSORS = [("blk.0.attn_q.weight", 4096, 4096), ("blk.0.attn_k.weight", 1024, 4096),
           ("blk.0.ffn_down.weight", 4096, 12288), ("blk.0.ffn_gate.weight", 12288, 4096),
           ("blk.1.attn_v.weight", 256, 192)]
SEED = 20260816


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    bad = 0
    for B in (1, 4):
        lay = tp.Layout(TENSORS, world, B)
        y_all = torch.zeros(B * lay.ysz, dtype=torch.float32, device=dev)
        descs, host = [], []
        for i, (n, N, K) in enumerate(TENSORS):
            tiles = synth.tiles_np(N, K, SEED + i)
            x = synth.x_np(K, B, SEED + 100 + i)
            shard = torch.from_numpy(np.ascontiguousarray(tp.shard_tiles(tiles, N, K, world, rank))).to(dev)
            descs.append({"tiles": shard, "x": torch.from_numpy(x).to(dev), "y": lay.local_view(y_all, i)})
            host.append((tiles, x))
        plan = q4rdna.Plan(descs, B=B)
        plan.run()
        gathered = torch.empty(world * B * lay.ysz, dtype=torch.float32, device=dev)
        tp.all_gather(y_all, gathered)
        torch.cuda.synchronize()
        own = y_all.cpu().numpy().copy()
        for i, y in enumerate(lay.assemble(gathered.cpu().numpy())):
            n, N, K = TENSORS[i]
            tiles, x = host[i]
            y64, mag = oracle.gemv_f64(tiles, x, N, K, threads=8)
            try:
                tolerance.check(y, y64, mag, f"rank {rank} B={B} {n}")
            except AssertionError as e:
                print(e, flush=True)
                bad += 1
            r0, rows = tp.shard_rows(N, world, rank)
            if not np.array_equal(y[:, r0:r0 + rows].view(np.uint32), lay.local_view(own, i).view(np.uint32)):
                print(f"rank {rank} B={B} {n}: own slice changed by the gather", flush=True)
                bad += 1
        # the fused gather: the same plan stores into every rank's gathered
        # buffer itself; both buffers (two runs) must equal the NCCL gather bit for bit
        want = gathered.cpu().numpy().view(np.uint32).copy()
        pg = tp.PeerGather(plan, lay, y_all)
        for run in range(3):
            for d, (tiles, x) in zip(descs, host):
                d["x"].copy_(torch.from_numpy(x))
            got = pg.run()
            torch.cuda.synchronize()
            if not np.array_equal(got.cpu().numpy().view(np.uint32), want):
                print(f"rank {rank} B={B} run {run}: fused gather differs from the NCCL gather", flush=True)
                bad += 1
        dist.barrier()
        pg.close()
        # dependent stages: two gather plans (the first tensors, the rest) run by
        # one q4rdna_plan_run_many call, which captures the pair once per run
        # parity and replays it, the flag exchange counting its epochs on the
        # device; four calls fill both gathered buffers twice
        stage_plans, pgs, wants = [], [], []
        for part in (TENSORS[:2], TENSORS[2:]):
            slay = tp.Layout(part, world, B)
            ys = torch.zeros(B * slay.ysz, dtype=torch.float32, device=dev)
            idx = [TENSORS.index(t) for t in part]
            sd = [{"tiles": descs[i]["tiles"], "x": descs[i]["x"], "y": slay.local_view(ys, k)}
                  for k, i in enumerate(idx)]
            sp = q4rdna.Plan(sd, B=B)
            sp.run()
            g = torch.empty(world * B * slay.ysz, dtype=torch.float32, device=dev)
            tp.all_gather(ys, g)
            torch.cuda.synchronize()
            wants.append(g.cpu().numpy().view(np.uint32).copy())
            pgs.append(tp.PeerGather(sp, slay, ys))
            stage_plans.append(sp)
        for run in range(4):
            q4rdna.run_plans(stage_plans)
            torch.cuda.synchronize()
            for k, (sp, spg) in enumerate(zip(stage_plans, pgs)):
                par = spg._lib.q4rdna_plan_gather_parity(sp._h)
                if not np.array_equal(spg.gathered[par].cpu().numpy().view(np.uint32), wants[k]):
                    print(f"rank {rank} B={B} run_many call {run} stage {k}: fused gather differs", flush=True)
                    bad += 1
        dist.barrier()
        for spg in pgs:
            spg.close()
        for sp in stage_plans:
            sp.close()
        plan.close()
        fault = q4rdna.take_fault()
        if fault:
            print(f"rank {rank}: device fault flag {fault}", flush=True)
            bad += 1
    flag = torch.tensor([bad], device=dev)
    dist.all_reduce(flag)
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print(f"tp parity world={world}: {'FAIL' if flag.item() else 'ok'}", flush=True)
    return 1 if flag.item() else 0


if __name__ == "__main__":
    sys.exit(main())
