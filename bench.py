#!/usr/bin/env python3
"""Benchmark: Q4_RDNA group-64 GEMV decode-step weight stream on B200.

Default workload (N=1): one Qwen3-8B decode step = 252 independent Q4 group-64
GEMVs (36 layers x q/k/v/o/gate/up/down, batch 1, fresh N(0,1) activation per
tensor), run as one multi-GEMV plan: one persistent-kernel launch per step, with
the split-K factor chosen for the whole plan (no split on the Qwen3-8B step).
The step streams 3.69 GB of packed weights, far more than L2 (126 MB), so no
L2 flush is needed between steps.

  value    aggregate HBM GB/s = algorithmic bytes of the step / device time
  e2e      same metric through the public C ABI with pinned HOST buffers: every
           step copies all 252 activations host->device and brings all outputs
           back (q4rdna_plan_run_host: the kernels store the outputs straight
           into the pinned buffer, and the input copies run in 2 graded
           segments overlapped with the GEMVs, so only the first segment's
           input copy is exposed; one CUDA graph replay per step)
  roofline dominant kernel (the plan kernel) vs MEASURED_PEAKS.json hbm_gbs
  cpu_baseline  the reference's own CPU GEMV (reference_q4_rdna compiled from
           its source into oracle/_ref) on the host cores, bounded sample

--gpus N (under torchrun): every tensor's output rows are sharded over the N
ranks (tensor parallel, rows in multiples of 32) and the y slices are gathered,
by default inside the plan kernel (P2P stores into every rank's gathered
buffer, then a flag exchange), or with one NCCL all-gather per step
(--gather nccl); total work is fixed (strong scaling).
--impl reference: the reference CPU implementation alone on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "rdna-gfx1201-v0.1_b200")
for _p in (REPO, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

FALLBACK_HBM_GBS = 6650.0
METRIC = "Q4-g64 GEMV HBM GB/s (% of peak) and us per Qwen3-8B decode step, 1/2/4/8 B200"
UNIT = "GB/s"


def hbm_peak():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        return float(json.load(open(p))["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic(workload: str):
    """Per-launch DRAM bytes of the plan kernel from the committed ncu summary."""
    p = os.path.join(REPO, "profiles", "q4_gemv_kernel_traffic.txt")
    if not os.path.exists(p):
        return None
    for line in open(p):
        line = line.strip()
        if line.startswith(workload + "="):
            try:
                return int(line.split("=", 1)[1].split()[0])
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 100 ms."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.proc is None or self.path is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in open(self.path):
            f = [c.strip() for c in line.split(",")]
            if len(f) >= 9:
                rows.append(f)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows),
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit()) if rows else None}


def cpu_count():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def reference_cpu_rate(budget_s: float, threads: int):
    """The reference's CPU GEMV (reference_q4_rdna, q4rdna_gemv_bench.hip:189-211,
    compiled unmodified from the reference file into oracle/_ref) run
    concurrently on `threads` host threads, each on its own 12288 x 4096 tensor
    (26.7 MB, so the working set exceeds the CPU caches), until `budget_s`
    seconds have passed.  Falls back to the oracle port (bit-exact with it) when
    oracle/_ref was not built.  Returns (GB/s, kind, threads, sample)."""
    import numpy as np

    import oracle
    from q4rdna import synth

    N, K = 12288, 4096
    nbytes = N * K * 34 // 64 + 4 * K + 4 * N
    pool = min(threads, 16)  # 16 x 26.7 MB distinct tensors: far above any CPU cache
    tiles = [synth.tiles_np(N, K, 31 + i) for i in range(pool)]
    xs = [synth.x_np(K, 1, 61 + i)[0] for i in range(threads)]
    kind = "reference" if oracle.ref is not None else "port"
    if kind == "reference":
        fns = [oracle.RefBenchGemv(t) for t in tiles]
        outs = [np.empty(N, np.float32) for _ in range(threads)]

    def one(i):
        if kind == "reference":
            # one prepared tensor per pool slot; y buffers are per call site
            ref = fns[i % pool]
            xv = xs[i]
            oracle.ref.q4ref_bench_run(ref._h, xv.ctypes.data_as(oracle._f32p), outs[i].ctypes.data_as(oracle._f32p))
        else:
            oracle.gemv_f32(tiles[i % pool], xs[i], N, K, threads=1, decode="refcpu")

    def round_():
        ts = [threading.Thread(target=one, args=(i,)) for i in range(threads)]
        for t in ts:
            t.start()
        for t in ts:
            t.join()

    round_()  # warm-up (page-in)
    calls, t0 = 0, time.perf_counter()
    while True:
        round_()
        calls += threads
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    sample = (f"reference_q4_rdna 12288x4096 f32 GEMV, {calls} calls on {threads} threads "
              f"({calls // threads} rounds, {el:.1f} s)")
    if kind == "port":
        sample = sample.replace("reference_q4_rdna", "oracle port of reference_q4_rdna")
    return calls * nbytes / el / 1e9, kind, threads, sample


def reference_pack_rate(threads: int):
    """The reference packer binary (q4rdna_sidecar_pack, compiled unmodified
    from the reference source into oracle/_ref, OpenMP over groups) packing one
    4096 x 4096 bf16 N(0, 0.02) tensor on `threads` host threads, wall clock.
    Returns (Gweights/s, sample) or (None, why)."""
    import numpy as np

    import oracle

    if not os.path.exists(oracle.REF_PACK_BIN):
        return None, "oracle/_ref/q4rdna_sidecar_pack not built"
    N, K = 4096, 4096
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    bits = ((w.view(np.uint32).astype(np.uint64) + 0x7FFF + ((w.view(np.uint32) >> 16) & 1)) >> 16).astype("<u2")
    with tempfile.TemporaryDirectory() as td:
        raw = os.path.join(td, "w.bin")
        bits.tofile(raw)
        man = os.path.join(td, "m.tsv")
        with open(man, "w") as f:
            f.write(f"{raw}\t0\t{N}\t{K}\tblk.0.attn_q.weight\n")
        env = dict(os.environ, OMP_NUM_THREADS=str(threads))
        t0 = time.perf_counter()
        subprocess.run([oracle.REF_PACK_BIN, man, os.path.join(td, "o.q4rdna")], check=True, env=env,
                       capture_output=True)
        el = time.perf_counter() - t0
    return N * K / el / 1e9, f"q4rdna_sidecar_pack, one 4096x4096 bf16 tensor, OpenMP on {threads} threads, {el:.2f} s"


def run_pack(args):
    """GPU packer throughput on the Qwen3-8B weight set: the 7 tensor shapes of
    a layer, bf16 N(0, 0.02) on the device, each packed once per layer (36 x 7 =
    252 tensors, 6.95 G weights), timed with CUDA events."""
    import torch

    import q4rdna
    from q4rdna import synth

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(args.seed)
    layer = [(N, K) for (_, N, K) in synth.model_tensors(args.model) if _.startswith("blk.0.")]
    nlayers = len(synth.model_tensors(args.model)) // len(layer)
    ws = [(torch.randn((N, K), generator=g, device=dev) * 0.02).to(torch.bfloat16) for N, K in layer]
    for w in ws:  # warm-up
        q4rdna.pack_bf16(w)
    torch.cuda.synchronize()
    l0 = q4rdna.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        e0.record()
        for _ in range(nlayers):
            for w in ws:
                q4rdna.pack_bf16(w)
        e1.record()
        torch.cuda.synchronize()
    sec = e0.elapsed_time(e1) / 1e3
    weights = nlayers * sum(N * K for N, K in layer)
    cpu = None
    if not args.no_cpu_baseline:
        v, sample = reference_pack_rate(cpu_count())
        if v is not None:
            cpu = {"value": round(v, 4), "unit": "Gweights/s", "cores": cpu_count(), "kind": "reference",
                   "sample": sample, "model_seconds": round(weights / (v * 1e9), 1)}
    return {"metric": f"Q4_RDNA sidecar packing of {args.model} (bf16 -> tiles), Gweights/s",
            "value": round(weights / sec / 1e9, 3), "unit": "Gweights/s", "model_seconds": round(sec, 3),
            "n_gpus": 1, "higher_is_better": True, "dtype": "bf16 in, int4 + fp16 scales out",
            "data": "synthetic: bf16 N(0, 0.02) weights of the model's shapes (no Qwen3 weights offline)",
            "config": {"workload": f"{nlayers} layers x {len(layer)} tensors, {weights} weights"},
            "cpu_baseline": cpu, "gpu_launches": q4rdna.launch_count() - l0, "clocks": clk.summary()}


# ------------------------------------------------- single drop-in calls

L2_BYTES = 126 * 1024 * 1024
# The reference's per-kernel medians (results/kernel_profile.json:46,51,56,
# RX 9070 XT, rocprofv3 trace of the split-K kernels) for the same shapes.
REF_MEDIAN_US = {"4096x4096": 16.88, "1024x4096": 5.40, "12288x4096 gate+up": 90.24}


def _time_graph(launch, n_launch: int, stream, reps: int = 7):
    """Median device us per launch: n_launch back-to-back launches captured in
    one CUDA graph on `stream`, replayed `reps` times between CUDA events."""
    import torch

    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(n_launch):
            launch(i)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ts = []
    for _ in range(reps):
        e0.record()
        g.replay()
        e1.record()
        e1.synchronize()
        ts.append(e0.elapsed_time(e1) * 1e3 / n_launch)
    del g
    return statistics.median(ts)


def run_single(args):
    """us per GEMV through the drop-in entry points, the way llama.cpp drives
    the reference (one launch per mul_mat node): configs 0 and 1 of the
    benchmark, plus the fused gate+up pair.  Each timing is `--single-launches`
    back-to-back calls captured in a CUDA graph and replayed (device time per
    call, no host overhead), rotating over enough weight copies to cover >= 4x
    L2 so every call streams its weights from HBM, as the reference's own
    benchmark rotates copies (q4rdna_gemv_bench.hip:137-161).  Legs:
      gemv       q4rdna_gemv (raw pointers, caller workspace), split from the
                 selector and forced to 1..16 (the split sweep);
      mul_mat    the name-keyed hooks q4rdna_mul_mat / q4rdna_mul_mat_glu on a
                 sidecar holding the copies (the selector's split)."""
    import ctypes

    import torch

    import q4rdna
    from q4rdna import synth

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L = q4rdna.lib
    if L is None:
        raise SystemExit("libq4rdna.so not built")
    peak, peak_kind = hbm_peak()
    shapes = [("4096x4096", 4096, 4096, q4rdna.OP_PLAIN), ("12288x4096", 12288, 4096, q4rdna.OP_PLAIN),
              ("4096x12288", 4096, 12288, q4rdna.OP_PLAIN), ("1024x4096", 1024, 4096, q4rdna.OP_PLAIN),
              ("12288x4096 gate+up", 12288, 4096, q4rdna.OP_SWIGLU)]
    if args.single_shapes:
        keep = set(args.single_shapes.split(","))
        shapes = [s for s in shapes if s[0] in keep]
    splits = [0] + (list(range(1, 17)) if args.single_sweep else [])
    cap = torch.cuda.Stream()  # warm-up and capture stream (the hooks keep a workspace per stream)
    rows = []
    l0 = q4rdna.launch_count()
    with ClockSampler(0) as clk:
        for si, (name, N, K, op) in enumerate(shapes):
            planes = 2 if op == q4rdna.OP_SWIGLU else 1
            tb = N * K * 34 // 64
            copies = max(2, -(-4 * L2_BYTES // (tb * planes)))
            W = [synth.tiles_torch(N, K, args.seed + 1000 * si + c, dev) for c in range(copies * planes)]
            x = torch.randn(K, generator=torch.Generator(device=dev).manual_seed(args.seed + si), device=dev)
            y = torch.empty(N, device=dev)
            algo = planes * tb + 4 * K + 4 * N
            if args.single_ncu:
                for i in range(3):  # three cold calls (distinct copies), no graph
                    c = i % copies
                    h = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
                    need = L.q4rdna_workspace_bytes(N, K, 1, op, None)
                    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=dev)
                    rc = (L.q4rdna_gemv_swiglu(W[2 * c].data_ptr(), W[2 * c + 1].data_ptr(), x.data_ptr(), y.data_ptr(),
                                               N, K, 1, None, ws.data_ptr(), need, h) if op == q4rdna.OP_SWIGLU else
                          L.q4rdna_gemv(W[c].data_ptr(), x.data_ptr(), y.data_ptr(), N, K, 1, None, ws.data_ptr(), need, h))
                    if rc != 0:
                        raise RuntimeError(f"{name}: status {rc}")
                torch.cuda.synchronize()
                rows.append({"shape": name, "N": N, "K": K, "leg": "ncu", "split": L.q4rdna_select_split(N, K, 1, op),
                             "selector": True, "us": 0.0, "algo_bytes": algo, "gbs": 0.0, "frac": 0.0})
                del W
                continue
            for split in splits:
                if split > K // 64:
                    continue
                cfg = q4rdna.Cfg()
                cfg.split = split
                need = L.q4rdna_workspace_bytes(N, K, 1, op, ctypes.byref(cfg))
                ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=dev)
                chosen = L.q4rdna_select_split(N, K, 1, op) if split == 0 else split

                def launch(i, cfg=cfg, need=need, ws=ws):
                    c = i % copies
                    h = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
                    if op == q4rdna.OP_SWIGLU:
                        rc = L.q4rdna_gemv_swiglu(W[2 * c].data_ptr(), W[2 * c + 1].data_ptr(), x.data_ptr(),
                                                  y.data_ptr(), N, K, 1, ctypes.byref(cfg), ws.data_ptr(), need, h)
                    else:
                        rc = L.q4rdna_gemv(W[c].data_ptr(), x.data_ptr(), y.data_ptr(), N, K, 1, ctypes.byref(cfg),
                                           ws.data_ptr(), need, h)
                    if rc != 0:
                        raise RuntimeError(f"q4rdna_gemv {name} split {split}: status {rc}")

                with torch.cuda.stream(cap):
                    for i in range(20):
                        launch(i)
                torch.cuda.synchronize()
                us = _time_graph(launch, args.single_launches, cap)
                rows.append({"shape": name, "N": N, "K": K, "leg": "gemv", "split": chosen,
                             "selector": split == 0, "us": round(us, 3), "algo_bytes": algo,
                             "gbs": round(algo / (us * 1e-6) / 1e9, 1), "frac": round(algo / (us * 1e-6) / 1e9 / peak, 4)})
                if split == 0:
                    # the same calls with programmatic dependent launch: each
                    # call's first weights stream while the previous one ends
                    cfg.flags = q4rdna.CFG_OVERLAP_PREVIOUS
                    us = _time_graph(launch, args.single_launches, cap)
                    cfg.flags = 0
                    rows.append({"shape": name, "N": N, "K": K, "leg": "gemv_overlap", "split": chosen,
                                 "selector": True, "us": round(us, 3), "algo_bytes": algo,
                                 "gbs": round(algo / (us * 1e-6) / 1e9, 1),
                                 "frac": round(algo / (us * 1e-6) / 1e9 / peak, 4)})
            if not args.single_no_hook and name in ("4096x4096", "1024x4096", "12288x4096 gate+up"):
                rows.append(_time_hook(args, name, N, K, op, W, copies, x, y, algo, peak, cap))
            del W
            torch.cuda.empty_cache()
    sel = {r["shape"]: r for r in rows if r["leg"] == "gemv" and r["selector"]}
    ovl = {r["shape"]: r for r in rows if r["leg"] == "gemv_overlap"}
    best = {}
    for r in rows:
        if r["leg"] == "gemv" and (r["shape"] not in best or r["us"] < best[r["shape"]]["us"]):
            best[r["shape"]] = r
    summary = {k: {"us": v["us"], "split": v["split"], "frac": v["frac"], "best_split": best[k]["split"],
                   "best_us": best[k]["us"], "us_overlapped": ovl[k]["us"] if k in ovl else None,
                   "reference_median_us": REF_MEDIAN_US.get(k)}
               for k, v in sel.items()}
    c0 = sel.get("4096x4096")
    return {"metric": "us per Q4-g64 GEMV through the drop-in entry points (batch 1), and HBM GB/s",
            "value": c0["us"] if c0 else None, "unit": "us", "higher_is_better": False, "n_gpus": 1,
            "dtype": "int4 x f32 (fp16 scales, f32 accumulate)",
            "data": "synthetic: uniform int4 codes, fp16 scales |N(0,1)|*0.003, x ~ N(0,1) f32",
            "config": {"workload": "configs 0 and 1: single GEMVs, batch 1, one launch per call",
                       "launches_per_timing": args.single_launches,
                       "l2": ">= 4x L2 of rotating weight copies per shape (no flush needed)",
                       "timing": "CUDA graph of back-to-back calls, CUDA events, median of 7 replays"},
            "peak": peak, "peak_kind": peak_kind, "summary": summary, "rows": rows,
            "gpu_launches": q4rdna.launch_count() - l0, "clocks": clk.summary()}


def _time_hook(args, name, N, K, op, W, copies, x, y, algo, peak, cap):
    """The name-keyed hooks on a sidecar that holds the rotating copies."""
    import ctypes

    import torch

    import q4rdna
    from q4rdna import format as fmt

    tmp = tempfile.mkdtemp(prefix="q4rdna_single_")
    path = os.path.join(tmp, "copies.q4rdna")
    if op == q4rdna.OP_SWIGLU:
        tensors = []
        for c in range(copies):
            tensors.append((f"blk.{c}.ffn_up.weight", W[2 * c].cpu().numpy(), N, K))
            tensors.append((f"blk.{c}.ffn_gate.weight", W[2 * c + 1].cpu().numpy(), N, K))
    else:
        suffix = "attn_output" if N == K else "attn_k"
        tensors = [(f"blk.{c}.{suffix}.weight", W[c].cpu().numpy(), N, K) for c in range(copies)]
    fmt.write_sidecar(path, tensors)
    L = q4rdna.lib
    q4rdna.registry_reset()
    os.environ["LLAMA_Q4_RDNA_SIDECAR"] = path
    os.environ.pop("LLAMA_Q4_RDNA_SCOPE", None)
    names = [t[0].encode() for t in tensors]

    def launch(i):
        c = i % copies
        h = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        if op == q4rdna.OP_SWIGLU:
            ok = L.q4rdna_mul_mat_glu(names[2 * c], K, N, names[2 * c + 1], K, N, x.data_ptr(), K, y.data_ptr(), N, h)
        else:
            ok = L.q4rdna_mul_mat(names[c], K, N, x.data_ptr(), K, y.data_ptr(), N, h)
        if ok != 1:
            raise RuntimeError(f"name-keyed hook fell back for {name}")

    with torch.cuda.stream(cap):  # loads the sidecar and this stream's workspace outside the capture
        for i in range(20):
            launch(i)
    torch.cuda.synchronize()
    us = _time_graph(launch, args.single_launches, cap)
    # host cost of one hook call (ctypes from Python: an upper bound of the C cost)
    torch.cuda.synchronize()
    with torch.cuda.stream(cap):
        t0 = time.perf_counter()
        for i in range(200):
            launch(i)
        host_us = (time.perf_counter() - t0) / 200 * 1e6
    torch.cuda.synchronize()
    q4rdna.registry_reset()
    os.environ.pop("LLAMA_Q4_RDNA_SIDECAR", None)
    os.unlink(path)
    os.rmdir(tmp)
    split = L.q4rdna_select_split(N, K, 1, op)
    return {"shape": name, "N": N, "K": K, "leg": "mul_mat_glu" if op == q4rdna.OP_SWIGLU else "mul_mat",
            "split": split, "selector": True, "us": round(us, 3), "algo_bytes": algo,
            "gbs": round(algo / (us * 1e-6) / 1e9, 1), "frac": round(algo / (us * 1e-6) / 1e9 / peak, 4),
            "host_us_per_call_python": round(host_us, 2)}


QKV = (".attn_q.", ".attn_k.", ".attn_v.")


def build_step(model: str, rank: int, world: int, device, seed: int, layers: int = 0, B: int = 1,
               norm: bool = False, hybrid: bool = False, split: int = 0):
    """Weights (this rank's row shard of every tensor), activations and outputs
    of one decode step, laid out by q4rdna.tp.Layout so that a step's inputs and
    outputs are each one contiguous buffer (one copy each way for the
    end-to-end leg, one all-gather for tensor parallelism).  hybrid: the
    reference's qkv-fallback scope (source/q4rdna.cu:685-691), attn_q/k/v in
    Q4_K (block_q4_K rows), every other tensor in Q4_RDNA."""
    import torch

    from q4rdna import synth, tp

    names = synth.model_tensors(model)
    if layers:
        names = [t for t in names if int(t[0].split(".")[1]) < layers]
    if hybrid:
        # the Q4_K tensors' activations and outputs first: one byte range each
        # way, disjoint from the Q4_RDNA segments', so that run_host overlaps
        # the Q4_K launch and its copies with the Q4_RDNA segments
        names = sorted(names, key=lambda t: 0 if any(q in t[0] for q in QKV) else 1)
    try:
        lay = tp.Layout(names, world, B=B)
    except ValueError as e:
        raise SystemExit(str(e))
    # tensor i: x block [B][K] at float B * (sum of earlier K), y block [B][rows]
    x_all = torch.empty(B * lay.xsz, dtype=torch.float32, device=device)
    y_all = torch.empty(B * lay.ysz, dtype=torch.float32, device=device)
    g = torch.Generator(device=device)
    g.manual_seed(seed)  # same activations on every rank (replicated x)
    x_all.normal_(generator=g)
    import q4rdna

    descs, xo = [], 0
    wbytes = abytes = nweights = 0
    for i, s in enumerate(lay.slots):
        # each rank draws its own shard (same distributions; the shard of one
        # full tensor is a byte slice, q4rdna.tp.shard_tiles)
        q4k = hybrid and any(q in names[i][0] for q in QKV)
        if q4k:
            t = synth.q4k_torch(s.rows, s.K, seed + 1 + i * world + rank, device)
            tb = synth.q4k_bytes(s.rows, s.K)
        else:
            t = synth.tiles_torch(s.rows, s.K, seed + 1 + i * world + rank, device)
            tb = s.rows * s.K * 34 // 64
        d = {"tiles": t, "x": x_all[B * xo:B * (xo + s.K)].view(B, s.K), "y": lay.local_view(y_all, i)}
        if split:
            d["split"] = split
        if q4k:
            d["format"] = q4rdna.FORMAT_Q4K
        if norm:  # x is the raw hidden state; the plan normalises it on the fly
            d["norm_weight"] = torch.ones(s.K, dtype=torch.float32, device=device)
            d["norm_eps"] = 1e-6
        descs.append(d)
        xo += s.K
        wbytes += tb
        nweights += s.rows * s.K
        abytes += tb + 4 * B * (s.K + s.rows)
    return descs, x_all, y_all, wbytes, abytes, len(names), lay, nweights


def step_bytes(model: str, B: int, layers: int = 0, hybrid: bool = False):
    """(tensors, weight bytes, algorithmic bytes, weights) of one whole decode
    step (all ranks together), from the model's shapes alone."""
    from q4rdna import synth

    names = synth.model_tensors(model)
    if layers:
        names = [t for t in names if int(t[0].split(".")[1]) < layers]
    wb = ab = nw = 0
    for name, N, K in names:
        tb = synth.q4k_bytes(N, K) if hybrid and any(q in name for q in QKV) else N * K * 34 // 64
        wb += tb
        ab += tb + 4 * B * (K + N)
        nw += N * K
    return len(names), wb, ab, nw


def step_config(args, world: int, p2p: bool):
    """The `config` object of the step's JSON line, shared by both arms."""
    ntensors, wbytes, abytes, nweights = step_bytes(args.model, args.batch, args.layers, args.hybrid)
    return {"workload": f"{args.model} decode-step weight stream: {ntensors} GEMVs batch {args.batch}"
                        + (f" (first {args.layers} layers only)" if args.layers else "")
                        + (", qkv-fallback hybrid: attn_q/k/v in Q4_K, the rest in Q4_RDNA" if args.hybrid else "")
                        + (f", rows sharded over {world} GPUs + " + ("all-gather fused into the plan kernel (P2P stores)"
                           if p2p else "NCCL all-gather") if world > 1 else ""),
            "tensors": ntensors, "batch": args.batch, "fused_rmsnorm": bool(args.norm),
            "flops_per_step": 2 * args.batch * nweights, "weight_bytes_per_step": wbytes,
            "algo_bytes_per_step": abytes, "parallelism": f"tp{world}" if world > 1 else "none",
            "l2": f"no flush: {wbytes / 1e9:.2f} GB streamed per step >> 126 MB L2"}


def time_drop_in_step(descs, B: int, steps: int, abytes: int, overlap: bool = False):
    """The step as len(descs) single q4rdna_gemv calls (one launch each, the
    selector's split per shape, one shared workspace), captured once in a CUDA
    graph and replayed `steps` times between CUDA events.  overlap: each call
    with Q4RDNA_CFG_OVERLAP_PREVIOUS (programmatic dependent launch)."""
    import ctypes

    import torch

    import q4rdna

    L = q4rdna.lib
    need = max(L.q4rdna_workspace_bytes(d["y"].shape[-1], d["x"].shape[-1], B, q4rdna.OP_PLAIN, None) for d in descs)
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=descs[0]["x"].device)
    cap = torch.cuda.Stream()
    cfg = q4rdna.Cfg()
    cfg.flags = q4rdna.CFG_OVERLAP_PREVIOUS if overlap else 0

    def step():
        h = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        for d in descs:
            N, K = d["y"].shape[-1], d["x"].shape[-1]
            rc = L.q4rdna_gemv(d["tiles"].data_ptr(), d["x"].data_ptr(), d["y"].data_ptr(), N, K, B,
                               ctypes.byref(cfg), ws.data_ptr(), need, h)
            if rc != 0:
                raise RuntimeError(f"q4rdna_gemv {N}x{K}: status {rc}")

    with torch.cuda.stream(cap):
        step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=cap):
        step()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        g.replay()
    e1.record()
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / steps
    peak, _ = hbm_peak()
    gbs = abytes / (us * 1e-6) / 1e9
    del g
    return {"how": f"{len(descs)} q4rdna_gemv calls per step (one launch each, selector split), one CUDA graph"
                   + (", programmatic dependent launch" if overlap else ""),
            "launches_per_step": len(descs), "us_per_step": round(us, 2), "gbs": round(gbs, 1),
            "frac": round(gbs / peak, 4)}


LAYER_STAGES = (("attn_q", "attn_k", "attn_v"), ("attn_output",), ("ffn_gate", "ffn_up"), ("ffn_down",))


def time_layered(args, descs, names, world, rank, B, p2p, steps, dev):
    """The step as a decoder runs it under tensor parallelism: per layer four
    dependent stages (q/k/v, o, gate/up, down), each one plan followed by its
    all-gather (fused into the plan with p2p, else one NCCL all-gather), in
    stream order.  The weights and activations are the step's; every stage has
    its own output and gathered buffers.  p2p: all stages' plans run through
    one q4rdna_plan_run_many call per step; NCCL: the stages are captured once
    in a CUDA graph.  Device time per step, max over ranks."""
    import torch
    import torch.distributed as dist

    import q4rdna
    from q4rdna import tp

    by_name = {n[0]: i for i, n in enumerate(names)}
    nlayers = len({n[0].split(".")[1] for n in names})
    plans, gathers, keep = [], [], []
    for L in range(nlayers):
        for stage in LAYER_STAGES:
            idx = [by_name[f"blk.{L}.{t}.weight"] for t in stage]
            lay = tp.Layout([names[i] for i in idx], world, B=B)
            y = torch.zeros(B * lay.ysz, dtype=torch.float32, device=dev)
            sd = [{"tiles": descs[i]["tiles"], "x": descs[i]["x"], "y": lay.local_view(y, k)} for k, i in enumerate(idx)]
            plan = q4rdna.Plan(sd, B=B)
            g = None
            if world > 1:
                g = tp.PeerGather(plan, lay, y) if p2p else torch.empty(world * y.numel(), device=dev)
            plans.append(plan)
            gathers.append(g)
            keep.append((sd, y))
    stream = torch.cuda.current_stream()
    graph = None
    if world > 1 and not p2p:
        cap = torch.cuda.Stream()

        def once():
            for plan, g, (_, y) in zip(plans, gathers, keep):
                plan.run()
                tp.all_gather(y, g)

        with torch.cuda.stream(cap):
            once()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=cap):
            once()

    def step():
        if graph is not None:
            graph.replay()
        else:
            q4rdna.run_plans(plans, stream)

    def timed():
        for _ in range(3):
            step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    ms = timed()
    ms_overlap = None
    if graph is None:
        # the same stages with programmatic dependent launch: each stage's
        # weights start streaming while the previous stage's kernels finish
        for plan in plans:
            plan.set_flags(q4rdna.CFG_OVERLAP_PREVIOUS)
        ms_overlap = timed()
    fault = q4rdna.take_fault()
    del graph
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    for plan, g in zip(plans, gathers):
        if isinstance(g, tp.PeerGather):
            g.close()
        plan.close()
    return {"how": f"{len(plans)} dependent plans per step ({len(LAYER_STAGES)} stages per layer), each followed by "
                   + ("its all-gather fused into the plan (P2P stores + flag exchange), one q4rdna_plan_run_many call"
                      if p2p else "one NCCL all-gather, captured in one CUDA graph") if world > 1 else
                   f"{len(plans)} dependent plans per step ({len(LAYER_STAGES)} stages per layer), no gather (one GPU)",
            "plans": len(plans), "us_per_step": round(ms * 1e3, 2),
            "us_per_step_overlapped": round(ms_overlap * 1e3, 2) if ms_overlap is not None else None,
            "fault_flags": fault}


def run_ours(args):
    import torch
    import torch.distributed as dist

    import q4rdna
    from q4rdna import tp

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpus != world:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    if q4rdna.lib is None:
        raise SystemExit("libq4rdna.so not built")

    B = args.batch
    if args.hybrid and args.norm:
        raise SystemExit("--hybrid takes no --norm (the Q4_K kernel has no fused RMSNorm)")
    emulate = args.emulate_world if world == 1 and args.emulate_world > 1 else 0
    if args.tp_layered and (args.hybrid or args.norm):
        raise SystemExit("--tp-layered runs the plain Q4_RDNA step (no --hybrid, no --norm)")
    descs, x_all, y_all, wbytes, abytes, ntensors, lay, nweights = build_step(
        args.model, rank if not emulate else 0, world if not emulate else emulate, dev, args.seed, args.layers, B,
        args.norm, args.hybrid, args.plan_split)
    plan = q4rdna.Plan(descs, B=B)
    plan.set_segments(args.run_segments)
    info = plan.info()
    stream = torch.cuda.current_stream()
    p2p = world > 1 and args.gather == "p2p" and not args.hybrid  # the fused gather has no Q4_K epilogue
    gathered = torch.empty(y_all.numel() * world, device=dev) if world > 1 and not p2p else None
    pg = tp.PeerGather(plan, lay, y_all) if p2p else None

    def run_plan():
        # p2p: the plan kernel stores into every rank's gathered buffer, then the flag exchange
        return pg.run(stream) if p2p else plan.run(stream)

    def step():
        out = run_plan()
        if world > 1 and not p2p:
            tp.all_gather(y_all, gathered)
            return gathered
        return out if p2p else y_all

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    barrier()
    k_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    l0 = q4rdna.launch_count()
    with ClockSampler(local) as clk:
        t0.record(stream)
        for i in range(args.steps):
            k_ev[i][0].record(stream)
            run_plan()
            k_ev[i][1].record(stream)
            if world > 1 and not p2p:
                tp.all_gather(y_all, gathered)
        t1.record(stream)
        barrier()
    launches = q4rdna.launch_count() - l0
    ms_total = t0.elapsed_time(t1)
    kern_ms = statistics.mean(a.elapsed_time(b) for a, b in k_ev)
    per_rank = None
    if world > 1:
        # the same plan without its gather on every rank: the plan kernel's own
        # time, and how far apart the ranks finish it (arrival skew)
        alone = q4rdna.Plan(descs, B=B)
        for _ in range(3):
            alone.run(stream)
        barrier()
        a_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for i in range(args.steps):
            a_ev[i][0].record(stream)
            alone.run(stream)
            a_ev[i][1].record(stream)
        barrier()
        alone_ms = statistics.mean(a.elapsed_time(b) for a, b in a_ev)
        alone.close()
        mine = torch.tensor([alone_ms, kern_ms], dtype=torch.float64, device=dev)
        allr = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(allr, mine)
        pa = [round(v[0].item() * 1e3, 2) for v in allr]
        pw = [round(v[1].item() * 1e3, 2) for v in allr]
        per_rank = {"plan_alone_us": pa, ("plan_with_gather_us" if p2p else "plan_us_before_nccl"): pw,
                    "plan_alone_skew_us": round(max(pa) - min(pa), 2),
                    "gather_cost_us": round(max(pw) - max(pa), 2) if p2p else None}
    q4k_leg = None
    if args.hybrid:
        # the Q4_K tensors alone, as one plan: the Q4_K kernel's own roofline
        kd = [d for d in descs if d.get("format") == q4rdna.FORMAT_Q4K]
        kplan = q4rdna.Plan(kd, B=B)
        kbytes = sum(d["tiles"].numel() + 4 * B * (d["x"].shape[-1] + d["y"].shape[-1]) for d in kd)
        for _ in range(max(3, args.warmup)):
            kplan.run(stream)
        barrier()
        kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for i in range(args.steps):
            kev[i][0].record(stream)
            kplan.run(stream)
            kev[i][1].record(stream)
        barrier()
        k_ms = statistics.mean(a.elapsed_time(b) for a, b in kev)
        kplan.close()
        kpk, _ = hbm_peak()
        q4k_leg = {"kernel": "q4k::q4k_gemv_kernel (plan of the Q4_K tensors alone)", "tensors": len(kd),
                   "algo_bytes": kbytes, "kernel_us": round(k_ms * 1e3, 2),
                   "achieved": round(kbytes / (k_ms * 1e-3) / 1e9, 1), "frac": round(kbytes / (k_ms * 1e-3) / 1e9 / kpk, 4),
                   "traffic": ncu_traffic(f"q4k_{args.model}_b{B}")}

    # the same step as llama.cpp drives the reference: one drop-in q4rdna_gemv
    # call per tensor (the selector's split, one shared workspace), captured
    # once in a CUDA graph and replayed
    drop_in = None
    if world == 1 and not args.hybrid and not args.norm:
        drop_in = time_drop_in_step(descs, B, args.steps, abytes)
        if B <= 2:
            drop_in["overlapped"] = time_drop_in_step(descs, B, args.steps, abytes, overlap=True)

    layered = None
    if args.tp_layered:
        names = [(s_.name, s_.N, s_.K) for s_ in lay.slots]
        layered = time_layered(args, descs, names, world, rank, B, p2p, args.steps, dev)
        layered["gbs"] = round(abytes * world / (layered["us_per_step"] * 1e-6) / 1e9, 1)

    # end-to-end: pinned host activations in, outputs out, every step.  Every
    # rank copies in the whole (replicated) activation and brings out its own
    # outputs: together the ranks' host buffers hold the whole step's result.
    x_host = torch.empty(x_all.numel(), dtype=torch.float32, pin_memory=True)
    x_host.copy_(x_all)
    y_host = torch.empty(y_all.numel(), dtype=torch.float32, pin_memory=True)

    def e2e_step():
        if world == 1 or p2p:
            # the public host-buffer entry point: input copies overlapped with the
            # GEMVs, outputs stored straight into the host buffer (with p2p also
            # into every rank's gathered buffer, then the flag exchange)
            plan.run_host(x_host, x_all, y_all, y_host, segments=args.segments, stream=stream)
            return
        x_all.copy_(x_host, non_blocking=True)
        step()
        y_host.copy_(y_all, non_blocking=True)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1)

    # max over ranks (device-timed)
    t = torch.tensor([ms_total, kern_ms, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_total, kern_ms, e2e_ms = t.tolist()
    total_algo = abytes * world  # identical shard sizes on every rank
    step_ms = ms_total / args.steps
    peak, peak_kind = hbm_peak()
    achieved = abytes / (kern_ms * 1e-3) / 1e9
    out = None
    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and not args.hybrid:
            v, kind, thr, sample = reference_cpu_rate(args.cpu_seconds, cpu_count())
            cpu = {"value": round(v, 3), "unit": UNIT, "cores": thr, "kind": kind, "sample": sample}
        out = {
            "metric": METRIC, "value": round(total_algo / (step_ms * 1e-3) / 1e9, 2), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 4),
            "us_per_step": round(step_ms * 1e3, 2), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int4 x f32 (fp16 scales, f32 accumulate)",
            "data": "synthetic: uniform int4 codes, fp16 scales |N(0,1)|*0.003, x ~ N(0,1) f32 (no Qwen3 weights offline)"
                    + ("; Q4_K tensors: uniform quant and 6-bit scale bytes, d and dmin fp16((0.5+|N(0,1)|)*2e-4)"
                       if args.hybrid else ""),
            "config": step_config(args, world, p2p) if not emulate else
                      {**step_config(args, 1, False), "emulated": f"rank 0 of {emulate}: its row shard of every tensor, "
                                                                  "no gather, on one GPU",
                       "algo_bytes_per_step": abytes, "weight_bytes_per_step": wbytes},
            "plan": {"items": info["items"], "grid": info["grid"], "split": args.plan_split or "plan-wide choice"},
            "e2e": {"value": round(total_algo / (e2e_ms / args.steps * 1e-3) / 1e9, 2), "unit": UNIT,
                    "us_per_step": round(e2e_ms / args.steps * 1e3, 2),
                    "h2d_bytes_per_step": x_all.numel() * 4 * world, "d2h_bytes_per_step": y_host.numel() * 4 * world,
                    **({"per_rank": "each rank: the whole activation in, its own outputs out"} if world > 1 else {})},
            "roofline": {"bound": "hbm", "kernel": q4rdna.kernel_name(B) + (" + q4k::q4k_gemv_kernel" if args.hybrid else "")
                         + (" (plan + fused gather)" if p2p else " (plan)"), "achieved": round(achieved, 1),
                         "peak": peak, "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "algo_bytes_per_launch": abytes, "kernel_us": round(kern_ms * 1e3, 2),
                         "traffic": ncu_traffic(f"{args.model}_tp{world}" + (f"_b{B}" if B > 1 else ""))},
            "cpu_baseline": cpu,
            "gpu_launches": launches,
            **({"drop_in_step": drop_in} if drop_in else {}),
            **({"per_rank": per_rank} if per_rank else {}),
            **({"layered": layered} if layered else {}),
            **({"q4k": q4k_leg} if q4k_leg else {}),
            "clocks": clk.summary(),
        }
    if pg is not None:
        torch.cuda.synchronize()
        dist.barrier()
        pg.close()
    plan.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return out


def run_reference(args):
    """The reference's own CPU GEMV on the host cores, on this arm's config.
    reference_q4_rdna (source/q4rdna_gemv_bench.hip:189-211) exists only at
    12288 x 4096 (ROWS, COLUMNS at :17-18), so each step times a bounded sample
    of the workload: that shape, which is the step's ffn_gate / ffn_up tensors
    (72 of the Qwen3-8B step's 252), one call per host thread at a time for
    --ref-step-seconds.  The rate is algorithmic GB/s like our arm's; the
    step-equivalent time is the whole step's bytes at that rate."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    world = int(os.environ.get("WORLD_SIZE", "1"))
    steps = []
    thr = cpu_count()
    for i in range(args.warmup + args.steps):
        v, kind, thr, sample = reference_cpu_rate(args.ref_step_seconds, thr)
        if i >= args.warmup:
            steps.append(v)
    v = statistics.mean(steps)
    cfg = step_config(args, world, world > 1 and args.gather == "p2p" and not args.hybrid)
    step_us = cfg["algo_bytes_per_step"] / (v * 1e9) * 1e6
    return {
        "metric": METRIC, "impl": "reference", "value": round(v, 3), "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32 (reference CPU GEMV)",
        "data": "synthetic: uniform int4 codes, fp16 scales |N(0,1)|*0.003, x ~ N(0,1) f32 (no Qwen3 weights offline)",
        "config": cfg,
        "us_per_step": round(step_us, 1),
        "sample": ("each step: " + sample + "; reference_q4_rdna is fixed at 12288x4096 "
                   "(q4rdna_gemv_bench.hip:17-18), the shape of the step's ffn_gate/ffn_up tensors; "
                   "us_per_step = the whole step's algorithmic bytes at the measured rate"),
        "cpu_baseline": {"value": round(v, 3), "unit": UNIT, "cores": thr, "kind": kind, "sample": sample},
        "e2e": {"value": round(v, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--model", choices=["qwen3-8b", "qwen3-32b"], default="qwen3-8b")
    ap.add_argument("--seed", type=int, default=20260816)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--ref-step-seconds", type=float, default=4.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--gather", choices=["p2p", "nccl"], default="p2p",
                    help="N > 1: all-gather fused into the plan kernel (p2p) or one NCCL all-gather per step")
    ap.add_argument("--pack", action="store_true",
                    help="time the GPU sidecar packer on the model's weights instead of the GEMV step")
    ap.add_argument("--norm", action="store_true",
                    help="every GEMV takes the raw hidden state and applies RMSNorm in the kernel (fused producer)")
    ap.add_argument("--run-segments", type=int, default=0,
                    help="device-resident step as this many overlapping launches (0 or 1: one launch)")
    ap.add_argument("--segments", type=int, default=0,
                    help="e2e leg at N = 1: plan segments whose host copies overlap the GEMVs (0: library default)")
    ap.add_argument("--batch", type=int, default=1,
                    help="activation columns per GEMV (1..16; 3..16 run the tile path)")
    ap.add_argument("--hybrid", action="store_true",
                    help="the reference's qkv-fallback scope: attn_q/k/v as Q4_K tensors, the rest Q4_RDNA")
    ap.add_argument("--single", action="store_true",
                    help="us per GEMV through the drop-in entry points (configs 0 and 1) instead of the step")
    ap.add_argument("--single-sweep", action="store_true", help="--single: also force split 1..16")
    ap.add_argument("--single-shapes", default="", help="--single: comma-separated subset of the shapes")
    ap.add_argument("--single-launches", type=int, default=1000, help="--single: calls per timed graph")
    ap.add_argument("--single-no-hook", action="store_true", help="--single: skip the name-keyed hook leg")
    ap.add_argument("--single-ncu", action="store_true",
                    help="--single: only 3 eager calls per shape at the selector's split (for an ncu launch list)")
    ap.add_argument("--plan-split", type=int, default=0,
                    help="force this split-K factor on every tensor of the step's plan (0: the plan-wide choice)")
    ap.add_argument("--emulate-world", type=int, default=0,
                    help="N = 1 only: run rank 0's row shards of a W-way split (no gather), e.g. for ncu")
    ap.add_argument("--tp-layered", action="store_true",
                    help="also time the step as 4 dependent plans per layer, each followed by its all-gather")
    ap.add_argument("--layers", type=int, default=0,
                    help="only the first L layers (small cases for profiling); 0 = the whole model")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    # stdout carries exactly one JSON line: library chatter (the NCCL version
    # banner, warnings) goes to stderr for the whole run
    sys.stdout.flush()
    result = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    if args.pack:
        out = run_pack(args)
    elif args.single:
        out = run_single(args)
    else:
        out = run_reference(args) if args.impl == "reference" else run_ours(args)
    if out is not None:
        print(json.dumps(out), file=result, flush=True)


if __name__ == "__main__":
    main()
