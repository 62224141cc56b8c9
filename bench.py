"""MoE stage forward benchmark on B200 (see --help).

Workload (all N): the V4-Flash-shaped MoE layer of config c1 (H=4096, 256 routed experts top-8,
I=2048, NVFP4 routed experts, FP8 128x128 shared expert, sigmoid router), verify chunks of M=16
tokens, 6 distinct layers per GPU. At N GPUs the 6N-layer stack is pipeline-partitioned into
contiguous 6-layer blocks, one per rank (N=8 is config c2's 48 layers), with NCCL send/recv of the
bf16 activations between stages and 16 chunks streamed per step (4 in flight per hop). Per-GPU work
is fixed: weak scaling.
Each layer runs as the reference block's ffn half, x + moe(rmsnorm(x)) (the residual add and the norm
fused in one kernel of this library), so the routing stays as spread deep in the stack as at its
first layer.

  value   = token-layers per second over the whole job: chunks * M tokens * layers / time, with
            the inputs already in HBM (one layer's MoE forward on M tokens = M token-layers; at N=1
            this is the single-layer c1 tokens/s at M=16).
  e2e     = the same through the public API with host buffers: every chunk is copied in from pinned
            host memory on stage 0 and its output read back to the host on the last stage.
  roofline = the grouped expert kernel (the w13 and w2 launches) on the headline workload, from CUDA
            events around its launches: algorithmic bytes (distinct routed experts' NVFP4 weights
            and scales + the shared expert) / time, against MEASURED_PEAKS.json's HBM copy figure.
  cpu_baseline = the CPU oracle (numpy restatement of the reference MoE.forward) on a sample of the
            same workload on the host cores.
  sweep   = (N=1) c1 at M = 1, 8, 32, 64 over the same 6 layers; one c3 layer (FP8 experts, Zipf
            selection) at M = 1, 16, 64 and one c4 layer (Kimi-K3-scale NVFP4, the prefill regime)
            at M = 256, 1024 under the default and each forced kernel choice (verify, prefill,
            hybrid), each forward starting from a flushed L2; fp8_gemm (the kernel seam's dense
            GEMM) at V4's attention / indexer / shared-expert shapes, M = 1 and 16.

--config c4 runs config c4's 61-layer stack instead (prefill chunks of M=256, split over the ranks
by even_tiling, strong scaling). --impl reference times the CPU path alone (rank 0), as the
reference arm.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

HEADLINE_M = 16
LAYERS_PER_GPU = 6
N_EXPERTS = None       # --experts: fewer routed experts per layer (the small case for ncu captures)
PREFILL = 0            # --prefill: expert-kernel choice of the tensor-core layout (0 by batch size)
# chunks per step: the timed region starts and ends with the pipeline empty (a barrier on each side),
# so N stages lose N-1 chunk times of fill and drain per timed region; 16 chunks a step keep that
# under 5% of 10 steps at 8 GPUs
CHUNKS_PER_STEP = 16
METRIC = "MoE stage tokens/s (token-layers/s), verify M=16, c1/c2 V4-Flash MoE layer"
# DRAM bytes (ncu dram__bytes_read.sum + dram__bytes_write.sum of one forward's W13 and W2 grouped
# launches) over that forward's algorithmic bytes, from one capture of the small case
# (--layers 1 --experts 32) per kernel family; roofline.traffic applies it to the live workload.
TRAFFIC_RATIO = {"tcgen05": (321.2 + 3.9 + 160.6 + 4.1) / 469.0, "mma.sync": (1.018e9 + 13.4e6 + 0.509e9 + 12.5e6) / 1.44e9}
UNIT = "tokens/s"


def env_int(k, d):
    try:
        return int(os.environ.get(k, d))
    except ValueError:
        return d


# ── peaks ────────────────────────────────────────────────────────────────────────────────────────

def hbm_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ── clocks ───────────────────────────────────────────────────────────────────────────────────────

class ClockSampler:
    """nvidia-smi clocks and throttle reasons every 50 ms; summary() keeps the samples taken inside
    the windows marked with region() (the timed regions)."""
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, path):
        self.path = path
        self.proc = None
        self.windows = []

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "50"], stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
            return self
        # nvidia-smi needs a moment to start sampling: wait for its first line
        t_end = time.time() + 5.0
        while time.time() < t_end and self.proc.poll() is None:
            self.f.flush()
            if os.path.getsize(self.path) > 0:
                break
            time.sleep(0.05)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.12)   # one more sample after the last window
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.f.close()

    class _Window:
        def __init__(self, owner):
            self.owner = owner

        def __enter__(self):
            self.t0 = time.time()

        def __exit__(self, *a):
            self.owner.windows.append((self.t0, time.time()))

    def region(self):
        return ClockSampler._Window(self)

    def summary(self, gpus):
        import datetime
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        rows = []
        with open(self.path) as f:
            for line in f:
                p = [x.strip() for x in line.split(",")]
                if len(p) < 10:
                    continue
                try:
                    ts = datetime.datetime.strptime(p[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                    idx = int(p[1])
                    rows.append((ts, idx, float(p[2]), float(p[3]), p[6:10]))
                except ValueError:
                    continue
        rows = [r for r in rows if r[1] in gpus]
        inside = [r for r in rows if any(t0 <= r[0] <= t1 for t0, t1 in self.windows)]
        if not inside and rows and self.windows:
            # windows shorter than the sampling interval: the samples nearest to each window
            inside = [min(rows, key=lambda r: min(abs(r[0] - t0) + abs(r[0] - t1) for t0, t1 in self.windows))]
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        reasons = set()
        for r in inside:
            for n, v in zip(names, r[4]):
                if v.lower() in ("active", "1"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(r[2] for r in inside), "sm_max_mhz": max(r[3] for r in inside),
                "samples": len(inside), "reasons": sorted(reasons)}


# ── workload ─────────────────────────────────────────────────────────────────────────────────────

def build_layers(rank, n_layers, device, cname="c1", first_layer=None, distinct=None):
    """This rank's layers of config `cname`. Layers past `distinct` alias the first `distinct`
    banks (a stack that does not fit in HBM cycles through as many distinct layers as fit; each bank
    is many times the L2, so every forward still streams its weights from HBM)."""
    from shard_b200 import synth as S
    cfg = S.CONFIGS[cname]
    if N_EXPERTS:
        cfg = cfg.replace(n_experts=N_EXPERTS)
    first = rank * n_layers if first_layer is None else first_layer
    nd = n_layers if distinct is None else max(1, min(distinct, n_layers))
    banks = [S.device_layer(cfg, layer=first + j, device=device, seeded=[], fill="normal", prefill=PREFILL)
             for j in range(nd)]
    return cfg, [banks[j % nd] for j in range(n_layers)]


def chunk_inputs(cfg, n, device, seed_step=0):
    from shard_b200 import synth as S
    xs = []
    for j in range(n):
        x, _ = S.make_inputs(cfg, HEADLINE_M, step=seed_step * 1000 + j)
        xs.append(x.to(device))
    return xs


def algorithmic_bytes(cfg, idx_list, m):
    """Per-forward algorithmic bytes: distinct routed experts + shared + gate + x in / y out."""
    from shard_b200 import formats as F
    h, i = cfg.hidden, cfg.inter
    per_e = F.weight_bytes(cfg.expert_fmt, 2 * i, h) + F.weight_bytes(cfg.expert_fmt, h, i)
    shared = F.weight_bytes(F.FMT_FP8, 2 * i, h) + F.weight_bytes(F.FMT_FP8, h, i) if cfg.n_shared else 0
    gate = cfg.n_experts * h * 2
    out = []
    for idx in idx_list:
        d = len(np.unique(idx))
        grouped = d * per_e + shared
        out.append((grouped, grouped + gate + 2 * m * h * 2))
    return out


def time_grouped(layers, cfg, m, reps=3):
    """CUDA events around the grouped kernel's launches (w13 + w2) of each layer, per forward."""
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
    for e in evs:
        e.record()
    torch.cuda.synchronize()
    rows = []
    xs = chunk_inputs(cfg, reps * len(layers), layers[0].device, seed_step=7)
    k = 0
    for r in range(reps):
        for lay in layers:
            y, idx, t = lay.forward_profiled(xs[k], evs)
            k += 1
            torch.cuda.synchronize()
            rows.append((idx.cpu().numpy(), t))
    return rows


def cpu_oracle_sample(cfg, n_tokens=2, layer=0, reps=1):
    """The CPU oracle on a bounded sample: n_tokens tokens of one c1 layer, all host threads."""
    from oracle import moe_oracle as O
    from shard_b200 import formats as F
    from shard_b200 import synth as S
    x, _ = S.make_inputs(cfg, HEADLINE_M, step=0)
    x = x[:n_tokens].float().numpy()
    gw, gb = S.make_gate(cfg, layer)
    _, idx, _ = O.gate(x, gw.float().numpy(), gb.numpy(), cfg.score_func, cfg.route_scale, cfg.topk)
    cache = {}
    for e in sorted(set(idx.ravel().tolist())):
        ew = S.make_expert(cfg, layer, e)
        cache[e] = tuple(t.numpy() for t in (ew.w13, ew.w13_s, ew.w13_ts, ew.w2, ew.w2_s, ew.w2_ts))
    sh = S.make_expert(cfg, layer, -1, F.FMT_FP8)
    lay = O.OracleLayer(hidden=cfg.hidden, inter=cfg.inter, topk=cfg.topk, score_func=cfg.score_func,
                        route_scale=cfg.route_scale, swiglu_limit=cfg.swiglu_limit, expert_fmt=cfg.expert_fmt,
                        gate_w=gw.float().numpy(), gate_b=gb.numpy(), expert=lambda e: cache[e],
                        shared=tuple(t.numpy() for t in (sh.w13, sh.w13_s, sh.w13_ts, sh.w2, sh.w2_s, sh.w2_ts)))
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        O.moe_forward(lay, x, workers=cores)
        ts.append(time.perf_counter() - t0)
    return n_tokens / min(ts), cores, f"c1 layer {layer}, {n_tokens} of the M={HEADLINE_M} chunk's tokens, " \
        f"{len(cache)} routed experts + shared, numpy fp32 dequant-then-matmul"


# ── arms ─────────────────────────────────────────────────────────────────────────────────────────

def run_reference(args, rank, world):
    if rank != 0:
        return 0
    from shard_b200 import synth as S
    cfg = S.CONFIGS["c1"]
    vals = []
    for s in range(args.warmup + args.steps):
        v, cores, sample = cpu_oracle_sample(cfg, n_tokens=1, layer=s % LAYERS_PER_GPU)
        if s >= args.warmup:
            vals.append(v)
    value = statistics.median(vals)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 / value,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,0.02) NVFP4 weights, N(0,1) bf16 tokens)",
            "config": {"workload": "c1 MoE layer, 1 token per step (bounded CPU sample)", "m": HEADLINE_M},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def run_gpu(args, rank, world, local_rank):
    import torch.distributed as dist
    from shard_b200.pipeline import Pipeline, StageStack

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    if args.config == "c4":
        return run_c4_pipeline(args, rank, world, device)
    cfg, layers = build_layers(rank, LAYERS_PER_GPU, device)
    pipe = Pipeline(StageStack(layers, residual=True), HEADLINE_M, cfg.hidden, rank, world, device, wire=args.wire)
    C = CHUNKS_PER_STEP
    xs_dev = chunk_inputs(cfg, C, device) if rank == 0 else None
    outs_dev = [torch.empty(HEADLINE_M, cfg.hidden, dtype=torch.bfloat16, device=device) for _ in range(C)] \
        if rank == world - 1 else None
    for lay in layers:
        lay.reserve(HEADLINE_M)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(step_fn, steps, warmup, clk=None):
        import contextlib
        for _ in range(warmup):
            step_fn()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with (clk.region() if clk is not None else contextlib.nullcontext()):
            e0.record()
            for _ in range(steps):
                step_fn()
            e1.record()
            torch.cuda.synchronize()
        barrier()
        return max_over_ranks(e0.elapsed_time(e1) / 1000.0)

    # device-resident value
    def step_dev():
        pipe.run(C, xs_dev, outs_dev)

    clk = ClockSampler(os.path.join(tempfile.gettempdir(), f"clocks_bench_r{rank}.csv"))   # scratch log
    clk.__enter__()   # sampling spans both timed regions (device-resident and end to end)
    t = timed(step_dev, args.steps, args.warmup, clk)
    tok_layers = args.steps * C * HEADLINE_M * LAYERS_PER_GPU * world
    value = tok_layers / t

    # end to end: pinned host in, pinned host out, through the public API
    xs_host = [x.cpu().pin_memory() for x in xs_dev] if rank == 0 else None
    outs_host = [torch.empty(HEADLINE_M, cfg.hidden, dtype=torch.bfloat16).pin_memory() for _ in range(C)] \
        if rank == world - 1 else None
    stage_in = [torch.empty(HEADLINE_M, cfg.hidden, dtype=torch.bfloat16, device=device) for _ in range(C)] \
        if rank == 0 else None

    def step_e2e():
        if rank == 0:
            for j in range(C):
                stage_in[j].copy_(xs_host[j], non_blocking=True)
        pipe.run(C, stage_in, outs_host)

    t_e2e = timed(step_e2e, args.steps, max(args.warmup, 3), clk)
    clk.__exit__(None, None, None)
    pipe.flush()
    torch.cuda.synchronize()
    e2e_value = tok_layers / t_e2e
    bytes_io = C * HEADLINE_M * cfg.hidden * 2

    # roofline of the grouped kernel on this rank's layers (rank 0 reports)
    roof = None
    sweep = {}
    if rank == 0:
        rows = time_grouped(layers, cfg, HEADLINE_M, reps=2)
        peak, kind = hbm_peak()
        nb = algorithmic_bytes(cfg, [r[0] for r in rows], HEADLINE_M)
        g_bytes = sum(b[0] for b in nb) / len(nb)
        g_time = sum(r[1]["grouped"] for r in rows) / len(rows)
        f_bytes = sum(b[1] for b in nb) / len(nb)
        f_time = sum(r[1]["total"] for r in rows) / len(rows)
        family = "tcgen05" if layers[0].layout == 1 else "mma.sync"
        kname = ("panel_kernel + tc_grouped_kernel" if family == "tcgen05" else "grouped_kernel") + \
            " (w13 and w2 launches of one forward)"
        roof = {"kernel": kname, "bound": "hbm",
                "achieved": g_bytes / g_time / 1e9, "peak": peak, "unit": "GB/s",
                "frac": g_bytes / g_time / 1e9 / peak,
                "traffic": g_bytes * TRAFFIC_RATIO[family],
                "traffic_basis": "ncu DRAM bytes / algorithmic bytes on the small capture case, times this "
                                 "workload's algorithmic bytes per forward",
                "peak_kind": f"{kind} (MEASURED_PEAKS.json hbm_gbs)" if kind == "measured" else "fallback",
                "algorithmic_bytes_per_forward": g_bytes, "grouped_us_per_forward": g_time * 1e6,
                "forward_us": f_time * 1e6, "forward_frac": f_bytes / f_time / 1e9 / peak,
                "phase_us": {k: sum(r[1][k] for r in rows) / len(rows) * 1e6
                             for k in ("route", "permute", "w13", "w2", "combine")}}
        if world == 1 and not args.no_sweep:
            sweep = m_sweep(layers, cfg)
            if not N_EXPERTS:
                sweep.update(cfg_sweep("c3", (1, 16, 64)))
                sweep.update(cfg_sweep("c4", (256, 1024), modes=(0, 1, 2, 3)))
                sweep.update(dense_sweep())
    clocks = clk.summary(set(range(world)) if world > 1 else {local_rank}) if rank == 0 else None
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        v, cores, sample = cpu_oracle_sample(cfg, n_tokens=2)
        cpu = {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample}
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": t / args.steps * 1000.0, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "nvfp4",
                "data": "synthetic (seeded N(0,0.02) weights quantised NVFP4 / FP8, N(0,1) bf16 tokens)",
                "config": {"workload": f"c1 MoE layer x {LAYERS_PER_GPU} per GPU, pipeline over {world} GPU(s) "
                                       f"({LAYERS_PER_GPU * world} layers; N=8 is c2's 48), M={HEADLINE_M} chunks",
                           "m": HEADLINE_M, "layers_per_gpu": LAYERS_PER_GPU, "chunks_per_step": C,
                           "hidden": cfg.hidden, "experts": cfg.n_experts, "topk": cfg.topk, "inter": cfg.inter,
                           "routed_fmt": "nvfp4", "shared_fmt": "fp8-128x128",
                           "kernels": "tcgen05" if layers[0].layout == 1 else "mma.sync",
                           "l2": "no flush: each step streams >1 GB of distinct expert weights per layer (L2 126 MB)",
                           "block": "x + moe(rmsnorm(x)) per layer (the reference block's ffn half; keeps routing "
                                    "spread through the stack)",
                           "parallelism": f"pp{world}", "wire": args.wire},
                "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": bytes_io,
                        "d2h_bytes_per_step": bytes_io},
                # per chunk and stage: 8 kernels per MoE forward on the verify path plus the fused
                # residual/RMSNorm before each layer and the final residual add; fp8 wire: a pack
                # and an unpack per stage boundary
                "gpu_launches": args.steps * C * ((LAYERS_PER_GPU * 9 + 1) * world +
                                                  (2 * (world - 1) if args.wire == "fp8" else 0)),
                "roofline": roof, "cpu_baseline": cpu, "clocks": clocks, "sweep": sweep}
        print(json.dumps(line), flush=True)
    return 0


C4_LAYERS = 61


def run_c4_pipeline(args, rank, world, device):
    """Config c4's stack: 61 Kimi-K3-scale layers (H=7168, 384 NVFP4 experts top-8, FP8 shared
    expert, Zipf routing) split over the ranks by even_tiling (8,8,8,8,8,7,7,7 at 8 GPUs), prefill
    chunks of M tokens (default 256) streamed through the stages. Strong scaling: the whole stack's
    work per step is fixed. value = tokens through all 61 layers per second (max over ranks)."""
    import datetime  # noqa: F401
    import torch.distributed as dist
    from shard_b200.pipeline import Pipeline, StageStack, even_tiling
    n_layers = args.c4_layers
    blocks = even_tiling(n_layers, world)
    mine = blocks[rank]
    free, _ = torch.cuda.mem_get_info(device)
    from shard_b200 import formats as F
    from shard_b200 import synth as S
    cfg0 = S.CONFIGS["c4"]
    per_layer = cfg0.n_experts * (F.weight_bytes(cfg0.expert_fmt, 2 * cfg0.inter, cfg0.hidden) +
                                  F.weight_bytes(cfg0.expert_fmt, cfg0.hidden, cfg0.inter)) * 2   # + staging
    distinct = args.distinct or max(1, int(0.6 * free // per_layer))
    cfg, layers = build_layers(rank, len(mine), device, "c4", first_layer=mine.start, distinct=distinct)
    m = args.m if args.m != HEADLINE_M else 256
    C = CHUNKS_PER_STEP
    for lay in layers:
        lay.reserve(m)
    pipe = Pipeline(StageStack(layers, residual=True), m, cfg.hidden, rank, world, device)
    xs = [S.make_inputs(cfg, m, step=j)[0].to(device) for j in range(C)] if rank == 0 else None
    outs = [torch.empty(m, cfg.hidden, dtype=torch.bfloat16, device=device) for _ in range(C)] \
        if rank == world - 1 else None

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[device.index])

    for _ in range(args.warmup):
        pipe.run(C, xs, outs)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    clk = ClockSampler(os.path.join(tempfile.gettempdir(), f"clocks_c4_r{rank}.csv"))
    clk.__enter__()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with clk.region():
        e0.record()
        for _ in range(args.steps):
            pipe.run(C, xs, outs)
        e1.record()
        torch.cuda.synchronize()
    barrier()
    clk.__exit__(None, None, None)
    t = e0.elapsed_time(e1) / 1000.0
    if world > 1:
        tt = torch.tensor([t], dtype=torch.float64, device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t = float(tt.item())
    pipe.flush()
    torch.cuda.synchronize()
    if rank == 0:
        tokens = args.steps * C * m
        line = {"metric": f"c4 MoE stack tokens/s ({n_layers} layers, prefill chunks)", "value": tokens / t,
                "unit": "tokens/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": t / args.steps * 1000.0, "higher_is_better": True, "scaling": "strong",
                "token_layers_per_s": tokens * n_layers / t, "dtype": "nvfp4", "data": "synthetic",
                "config": {"workload": f"c4 {n_layers}-layer MoE stack, pp{world} (even_tiling: "
                                       f"{[len(b) for b in blocks]}), M={m} chunks, {C} chunks per step",
                           "m": m, "layers": n_layers, "layers_per_rank": [len(b) for b in blocks],
                           "distinct_banks_per_rank": min(distinct, len(mine)), "chunks_per_step": C,
                           "pipeline_depth": pipe.depth, "parallelism": f"pp{world}",
                           "block": "x + moe(rmsnorm(x)) per layer",
                           "l2": "no flush: each forward streams GBs of distinct expert weights"},
                "clocks": clk.summary(set(range(world)) if world > 1 else {device.index})}
        print(json.dumps(line), flush=True)
    return 0


def m_sweep(layers, cfg):
    """c1 at M in {1, 8, 32, 64}: tokens/s per layer and the grouped kernel's HBM fraction."""
    peak, _ = hbm_peak()
    out = {}
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
    for e in evs:
        e.record()
    from shard_b200 import synth as S
    for m in (1, 8, 32, 64):
        xs = [S.make_inputs(cfg, m, step=500 + j)[0].to(layers[0].device) for j in range(len(layers))]
        for lay in layers:
            lay.reserve(m)
        for lay, x in zip(layers, xs):
            lay.forward(x)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 5
        e0.record()
        for _ in range(reps):
            for lay, x in zip(layers, xs):
                lay.forward(x)
        e1.record()
        torch.cuda.synchronize()
        t_fwd = e0.elapsed_time(e1) / 1000.0 / (reps * len(layers))
        rows = []
        for lay, x in zip(layers, xs):
            y, idx, t = lay.forward_profiled(x, evs)
            torch.cuda.synchronize()
            rows.append((idx.cpu().numpy(), t))
        nb = algorithmic_bytes(cfg, [r[0] for r in rows], m)
        g = sum(b[0] for b in nb) / sum(r[1]["grouped"] for r in rows) / 1e9
        f = sum(b[1] for b in nb) / len(nb) / t_fwd / 1e9
        out[f"c1_m{m}"] = {"tokens_per_s": m / t_fwd, "forward_us": t_fwd * 1e6, "grouped_gbs": g,
                           "grouped_frac": g / peak, "forward_gbs": f, "forward_frac": f / peak}
    return out


def cfg_sweep(name, ms, reps=4, modes=(0,)):
    """One layer of config `name` (c3: FP8 experts, Zipf selection, no shared expert; c4: Kimi-K3-scale
    NVFP4 prefill) at each M: every timed forward gets fresh tokens and starts with L2 flushed
    (a 256 MB write outside the timed region), since a single layer's active experts can be close to
    the 126 MB L2 at small M. modes: expert-kernel choices timed (0 the default choice, keyed
    `<name>_m<M>`; 1 the verify kernel, 2 the prefill kernel and 3 the hybrid dispatch, keyed with a
    suffix)."""
    from shard_b200 import synth as S
    peak, _ = hbm_peak()
    cfg = S.CONFIGS[name]
    lay = S.device_layer(cfg, layer=0, device=torch.device("cuda", torch.cuda.current_device()), seeded=[],
                         fill="normal")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=lay.device)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
    for e in evs:   # recorded once through torch, so torch accepts the C ABI's later records
        e.record()
    out = {}
    for m, mode in [(m, mode) for m in ms for mode in modes]:
        lay.prefill = mode
        lay.reserve(m)
        xs = [S.make_inputs(cfg, m, step=900 + r)[0].to(lay.device) for r in range(reps + 1)]
        lay.forward(xs[-1])
        t_fwd, rows = 0.0, []
        for r in range(reps):
            flush.fill_(r & 0xFF)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            lay.forward(xs[r])
            e1.record()
            torch.cuda.synchronize()
            t_fwd += e0.elapsed_time(e1) / 1000.0 / reps
            flush.fill_((r + 7) & 0xFF)
            y, idx, t = lay.forward_profiled(xs[r], evs)
            torch.cuda.synchronize()
            rows.append((idx.cpu().numpy(), t))
        nb = algorithmic_bytes(cfg, [r_[0] for r_ in rows], m)
        g = sum(b[0] for b in nb) / sum(r_[1]["grouped"] for r_ in rows) / 1e9
        f = sum(b[1] for b in nb) / len(nb) / t_fwd / 1e9
        key = f"{name}_m{m}" + {0: "", 1: "_verify", 2: "_prefill", 3: "_hybrid"}[mode]
        out[key] = {"tokens_per_s": m / t_fwd, "forward_us": t_fwd * 1e6, "grouped_gbs": g,
                    "grouped_frac": g / peak, "forward_gbs": f, "forward_frac": f / peak,
                    "l2": "flushed before each forward"}
    del lay, flush
    torch.cuda.empty_cache()
    return out


# V4-Flash's dense FP8 projections that decode runs through model.linear -> fp8_gemm, [N, K]
# (engines/deepseek_v4/v4_fp8_gemv.py:9-13): attention and indexer projections, shared expert.
V4_DENSE = [("wq_a", 1024, 4096), ("wkv", 512, 4096), ("wo_b", 4096, 8192), ("wq_b", 32768, 1024),
            ("idx_wq_b", 8192, 1024), ("shared_w1", 2048, 4096), ("shared_w2", 4096, 2048)]


def dense_sweep(ms=(1, 16)):
    """fp8_gemm (sb_qgemm, FP8 128x128 block scales, the tensor-core layout) at the V4 dense shapes, as
    a decode step runs them: a CUDA graph of back-to-back calls, each on its own copy of the weights
    (the copies together exceed the 126 MB L2, so every call streams its weights from HBM), replayed
    and timed with CUDA events; `us` = device time per call. Bytes moved per call (weights + scales +
    activations + output) per second against the measured HBM peak."""
    from shard_b200 import _lib, formats as F, ops
    from shard_b200.moe import tile
    peak, _ = hbm_peak()
    L = _lib.lib()
    dev = torch.device("cuda", torch.cuda.current_device())
    out = {}
    for name, n, k in V4_DENSE:
        g = torch.Generator().manual_seed(n * 7 + k)
        w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
        p, sc = F.quant_fp8_block(w)
        wt, wst = tile(F.FMT_FP8, _lib.MAT_PLAIN, p.view(torch.uint8).to(dev), sc.float().to(dev), 1, n, k,
                       _lib.LAYOUT_TC)
        copies = max(2, min(128, -(-(256 << 20) // wt.numel())))
        wts = [wt] + [wt.clone() for _ in range(copies - 1)]
        for m in ms:
            x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(dev)
            q, s = ops.act_quant(x, 128, "ue8m0")
            s = s.float().contiguous()
            y = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
            wsb = L.sb_qgemm_workspace_bytes(F.FMT_FP8, _lib.LAYOUT_TC, n, k, m)
            ws = torch.empty(max(wsb, 256), dtype=torch.uint8, device=dev)

            def calls():
                st = _lib.stream_ptr()
                for wc in wts:
                    _lib.check(L.sb_qgemm(F.FMT_FP8, _lib.LAYOUT_TC, wc.data_ptr(), wst.data_ptr(), None, n, k,
                                          q.data_ptr(), s.data_ptr(), m, y.data_ptr(), ws.data_ptr(), wsb, st),
                               "sb_qgemm")
            calls()
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                with torch.cuda.graph(graph, stream=side):
                    calls()
            torch.cuda.current_stream().wait_stream(side)
            graph.replay()
            torch.cuda.synchronize()
            ts = []
            for _ in range(3):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                graph.replay()
                e1.record()
                torch.cuda.synchronize()
                ts.append(e0.elapsed_time(e1) * 1000.0 / copies)
            del graph
            us = sorted(ts)[1]
            nbytes = n * k + (n // 128) * (k // 128) * 4 + m * k + m * (k // 128) * 4 + m * n * 2
            gbs = nbytes / (us * 1e-6) / 1e9
            out[f"fp8_gemm_{name}_m{m}"] = {"n": n, "k": k, "m": m, "us": us, "gbs": gbs, "frac": gbs / peak,
                                            "weight_copies": copies,
                                            "l2": "rotating weight copies > L2, graph-replayed back to back"}
        del wts
        torch.cuda.empty_cache()
    return out


def main():
    global LAYERS_PER_GPU, N_EXPERTS, HEADLINE_M, PREFILL
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--layers", type=int, default=LAYERS_PER_GPU,
                    help="layers per GPU (a smaller stack is the small case for ncu captures)")
    ap.add_argument("--experts", type=int, default=None,
                    help="routed experts per layer (default c1's 256; fewer is the small case for ncu captures)")
    ap.add_argument("--wire", choices=["bf16", "fp8"], default="bf16",
                    help="stage-boundary activation wire at N > 1 (fp8: the reference's e4m3 + per-row scale)")
    ap.add_argument("--layout", choices=["tc", "fragment"], default=None,
                    help="weight layout / kernel family (default: the library default)")
    ap.add_argument("--m", type=int, default=HEADLINE_M,
                    help="tokens per chunk (default 16, the headline; larger M with fewer --experts is the "
                         "small case for ncu captures of the prefill kernel)")
    ap.add_argument("--prefill", type=int, choices=[0, 1, 2, 3], default=0,
                    help="expert kernels on the tensor-core layout: 0 by batch size, 1 verify, 2 prefill, "
                         "3 hybrid dispatch")
    ap.add_argument("--config", choices=["c1", "c4"], default="c1",
                    help="c1: the headline (c1 layers, verify chunks, weak scaling); c4: the 61-layer "
                         "Kimi-K3-scale stack split over the GPUs with prefill chunks (--m, default 256)")
    ap.add_argument("--distinct", type=int, default=None,
                    help="c4: distinct layer banks per rank (default: as many as fit in 60%% of free HBM)")
    ap.add_argument("--c4-layers", type=int, default=C4_LAYERS,
                    help="c4: layers of the stack (default 61; a shorter stack is the small case for "
                         "launch-list captures)")
    args = ap.parse_args()
    if args.layout is not None:
        import shard_b200.moe as sbm
        from shard_b200 import _lib
        sbm.DEFAULT_LAYOUT = _lib.LAYOUT_TC if args.layout == "tc" else _lib.LAYOUT_FRAGMENT
    args.warmup = max(args.warmup, 3)
    LAYERS_PER_GPU = args.layers
    N_EXPERTS = args.experts
    HEADLINE_M = args.m
    PREFILL = args.prefill
    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local_rank = env_int("LOCAL_RANK", 0)
    if args.impl == "reference":
        return run_reference(args, rank, world)
    import datetime
    import torch.distributed as dist
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        return run_gpu(args, rank, world, local_rank)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
