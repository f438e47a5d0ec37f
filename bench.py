#!/usr/bin/env python
"""Benchmark: Stable Audio 3 medium DiT denoiser step (FP8 linears) on B200.

One step = one DiffusionTransformer.forward of the rf_denoiser with CFG
(cond + uncond halves batched) at the medium shape: dim 1536, 24 blocks,
24 heads x 64, differential attention, window (256, 256), L = 8183 latent
tokens (+64 memory tokens), 128 context tokens, FP8 e4m3 linears with
per-output-channel weight scales and per-tensor dynamic activation scales,
random-init weights (no checkpoints offline), synthetic N(0,1) latents.

Metric: latent tokens/s = (sum over sequences in the step, both CFG halves, of
L) / step time; the per-step latency is reported as ms_per_step. Every
rank of a torchrun launch runs its own prompt (data-parallel, weak scaling,
no collective in the step); value = all ranks' tokens / max-over-ranks time.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]
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
sys.path.insert(0, os.path.join(ROOT, "stable-audio-3_b200"))

import torch  # noqa: E402

WORKLOADS = {
    # the headline configuration: medium DiT, FP8 linears, L = 8183, one prompt = one CFG pair per GPU
    "medium_fp8": dict(model="medium", mode="fp8", L=8183, prompts=1, Tc=128, cfg_scale=7.0, apg_scale=1.0),
    # medium DiT with GPTQ int4 weight-only linears (group 128, act-order), L = 2584, batch 16 (8 CFG pairs)
    "medium_gptq": dict(model="medium", mode="gptq", L=2584, prompts=8, Tc=128, cfg_scale=7.0, apg_scale=1.0),
    # data-parallel sweep: 256 prompts, lengths ~ U{108..8183}, each with a CFG pair, LPT-sharded over the
    # ranks and packed variable-length (no padding) in batches of <= 2^18 token rows; one step = one
    # denoiser step over every prompt
    "dp_varlen_fp8": dict(model="medium", mode="fp8", dp=True, n_prompts=256, len_lo=108, len_hi=8183, Tc=128,
                          cfg_scale=7.0, apg_scale=1.0, max_tokens=1 << 18),
    # one long sequence split over the ranks: L = 16384 (+64 memory tokens on rank 0), one CFG pair, contiguous
    # token ranges per rank, +-256-row halos of q|k|v exchanged over NCCL before every self-attention
    "seq_split_fp8": dict(model="medium", mode="fp8", seq_split=True, L=16384, Tc=128, cfg_scale=7.0, apg_scale=1.0),
    # small DiT in bf16 (24 blocks, dim 1024, L = 2584, CFG pair)
    "small_bf16": dict(model="small", mode="bf16", L=2584, prompts=1, Tc=128, cfg_scale=7.0, apg_scale=1.0),
}
METRIC = "Medium DiT step latency (ms) + latent tokens/s at 1/2/4/8 B200, FP8/GPTQ"
UNIT = "latent tokens/s"


def _profiled_traffic(name):
    """dram__bytes_read + dram__bytes_write of one launch, from the committed ncu summary of that kernel."""
    try:
        for line in open(os.path.join(ROOT, "profiles", name)):
            if line.startswith("traffic_bytes_per_launch:"):
                return int(line.split(":")[1])
    except OSError:
        pass
    return None


def _peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9 or not f[0].isdigit() or int(f[0]) != self.idx:
                continue
            rows.append(f)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        loaded = [s for s in sm if mx and s > 0.5 * max(mx)] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_over_ranks(v: float, world: int) -> list:
    """Every rank's value, in rank order (same collective on every rank)."""
    if world == 1:
        return [v]
    import torch.distributed as dist
    t = torch.tensor([v], device="cuda", dtype=torch.float64)
    out = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(x.item()) for x in out]


def model_cfg(name):
    from sa3_b200.modules import MEDIUM, SMALL
    return {"medium": MEDIUM, "small": SMALL}[name]


def make_inputs(wl, cfg, seed, device):
    g = torch.Generator().manual_seed(seed)
    P, L = wl.get("prompts", 1), wl["L"]
    x = torch.randn(P, cfg.io_channels, L, generator=g)
    t = torch.full((P,), 0.5)
    cond = torch.randn(P, wl["Tc"], cfg.cond_token_dim, generator=g)
    gemb = torch.randn(P, cfg.global_cond_dim, generator=g)
    loc = torch.zeros(P, cfg.local_add_cond_dim, L)
    return [a.to(device) if device is not None else a for a in (x, t, cond, gemb, loc)]


# ----------------------------------------------------------------------------- CPU baseline (oracle port)
_CPU_MODEL = {}


def cpu_dit_sample(wl, threads: int, latents: int = 0):
    """Time the oracle's fp32 restatement of a one-block DiT forward (prologue MLPs, project_in, one full
    block with self- and cross-attention, local conditioning and FF, project_out) for ONE sequence of
    `latents` latents (default: the workload's full L) on the host cores. FP8 workloads use the oracle's
    FP8 definition (fake-quantized activations, e4m3 weights); GPTQ and bf16 workloads use fp32 linears
    (the dequantised GPTQ weight costs the same GEMM). A step is `depth` blocks over 2 CFG halves per
    prompt, so the sample is scaled by depth x 2 x prompts x L / latents (the prologue and projections
    are a few percent of one block, and are counted once per block: the figure errs on the slow side).
    Returns (seconds per full step, seconds measured, latents)."""
    from oracle import dit as odit
    from sa3_b200.modules import DiffusionTransformer, init_synthetic_, with_depth
    torch.set_num_threads(threads)
    cfg = model_cfg(wl["model"])
    key = wl["model"]
    if key not in _CPU_MODEL:
        sd = init_synthetic_(DiffusionTransformer(with_depth(cfg, 1)), seed=0).state_dict()
        _CPU_MODEL[key] = {k: v.float() for k, v in sd.items()}
    sd = _CPU_MODEL[key]
    mode = "fp8" if wl["mode"] == "fp8" else "fp32"
    if (key, mode) not in _CPU_MODEL:  # weights are quantized once, as a deployed CPU path would keep them
        _CPU_MODEL[(key, mode)] = odit.Linears(sd, mode)
    lin = _CPU_MODEL[(key, mode)]
    oc = odit.Cfg(io_channels=cfg.io_channels, embed_dim=cfg.embed_dim, depth=1, num_heads=cfg.num_heads,
                  cond_token_dim=cfg.cond_token_dim, global_cond_dim=cfg.global_cond_dim,
                  local_add_cond_dim=cfg.local_add_cond_dim, num_memory_tokens=cfg.num_memory_tokens,
                  sliding_window=cfg.sliding_window, differential=cfg.differential, ff_mult=cfg.ff_mult)
    n = min(latents, wl["L"]) if latents else wl["L"]
    g = torch.Generator().manual_seed(1)
    x = torch.randn(1, cfg.io_channels, n, generator=g)
    t = torch.full((1,), 0.5)
    cond = torch.randn(1, wl["Tc"], cfg.cond_token_dim, generator=g)
    gemb = torch.randn(1, cfg.global_cond_dim, generator=g)
    loc = torch.zeros(1, cfg.local_add_cond_dim, n)
    with torch.inference_mode():
        t0 = time.perf_counter()
        odit.dit_inner_forward(lin, sd, oc, x, t, cond, gemb, loc)
        dt = time.perf_counter() - t0
    return dt * cfg.depth * 2 * wl.get("prompts", 1) * (wl["L"] / n), dt, n


def _cpu_sample_text(wl, n, meas=None):
    cfg = model_cfg(wl["model"])
    lin = "FP8-definition" if wl["mode"] == "fp8" else "fp32"
    m = f" ({meas:.1f} s measured)" if meas is not None else ""
    scale = "" if n == wl["L"] else f" x{wl['L']}/{n} latents"
    return (f"oracle fp32 one-block {wl['model']} DiT ({lin} linears; self+cross attention, local cond, FF, "
            f"projections) over one sequence of {n} latents{m}, scaled x{cfg.depth} blocks x2 CFG halves"
            f"{' x' + str(wl.get('prompts', 1)) + ' prompts' if wl.get('prompts', 1) > 1 else ''}{scale}")


REFERENCE_SAMPLE_LATENTS = 2048


def run_reference(args, wl, world, rank):
    """The reference arm: the oracle port (the reference is Python; nothing compiles) on all host cores.
    Each step is a bounded sample: the one-block DiT over REFERENCE_SAMPLE_LATENTS latents."""
    if rank != 0:
        return
    if "L" not in wl:
        wl = dict(wl, L=8183, prompts=1)
    threads = len(os.sched_getaffinity(0))
    tokens = 2 * wl["L"] * wl.get("prompts", 1)
    for _ in range(args.warmup):
        cpu_dit_sample(wl, threads, REFERENCE_SAMPLE_LATENTS)
    steps = []
    n = REFERENCE_SAMPLE_LATENTS
    for _ in range(args.steps):
        s_step, _dt, n = cpu_dit_sample(wl, threads, REFERENCE_SAMPLE_LATENTS)
        steps.append(s_step)
    step_s = statistics.median(steps)
    value = tokens / step_s
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "L": wl["L"], "prompts_per_gpu": wl.get("prompts", 1),
                   "parallelism": f"dp{world}"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": _cpu_sample_text(wl, n)},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ----------------------------------------------------------------------------- peaks and rooflines
def measured_fp8_peak(dev) -> tuple:
    """Dense FP8 e4m3 GEMM throughput of the library path on this GPU (cuBLASLt through torch._scaled_mm,
    8192^3, per-tensor scales, bf16 out), best of 10 with CUDA events: the FP8 counterpart of the driver's
    measured cuBLAS bf16 figure. Returns (TFLOP/s, source text) or (None, reason)."""
    try:
        n = 8192
        a = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn)
        b = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn)
        one = torch.ones((), device=dev)
        f = lambda: torch._scaled_mm(a, b.t(), scale_a=one, scale_b=one, out_dtype=torch.bfloat16)  # noqa: E731
        for _ in range(3):
            f()
        torch.cuda.synchronize()
        best = float("inf")
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for _ in range(10):
            e0.record()
            f()
            e1.record()
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1))
        del a, b
        return 2.0 * n ** 3 / (best / 1e3) / 1e12, "measured here: torch._scaled_mm e4m3 8192^3 (cuBLASLt), best of 10"
    except Exception as exc:  # an image without the FP8 library path
        return None, f"fp8 library GEMM unavailable ({type(exc).__name__})"


def band_pairs(n: int, wl: int, wr: int) -> int:
    """Visible (query, key) pairs of a length-n sequence under a (wl, wr) band (negative = unbounded)."""
    import numpy as np
    i = np.arange(n)
    hi = np.full(n, n - 1) if wr < 0 else np.minimum(n - 1, i + wr)
    lo = np.zeros(n, dtype=np.int64) if wl < 0 else np.maximum(0, i - wl)
    return int((hi - lo + 1).sum())


def score_tiles(n: int, wl: int, wr: int, bm: int = 128, bn: int = 128) -> int:
    """128 x 128 score tiles the attention kernel computes for one head of one length-n sequence: each
    128-query tile visits the key tiles from its first visible key to its last (fully masked tiles skipped)."""
    t = 0
    for i0 in range(0, n, bm):
        i1 = min(i0 + bm, n) - 1
        lo = 0 if wl < 0 else max(0, i0 - wl)
        hi = n if wr < 0 else min(n, i1 + wr + 1)
        t += (hi - lo + bn - 1) // bn if hi > lo else 0
    return t


# ----------------------------------------------------------------------------- our arm
def run_dp_varlen(args, wl, world, rank, local):
    """Variable-length data-parallel sweep (no collective in the step; max-over-ranks device time)."""
    import numpy as np

    from sa3_b200 import dist as sdist
    from sa3_b200.modules import DiffusionTransformer, init_synthetic_

    dev = torch.device("cuda", local)
    cfg = model_cfg(wl["model"])
    model = init_synthetic_(DiffusionTransformer(cfg), seed=0).quantize(wl["mode"])
    eng = model.engine()
    rng = np.random.default_rng(0)
    lengths = [int(x) for x in rng.integers(wl["len_lo"], wl["len_hi"] + 1, size=wl["n_prompts"])]
    shard = sdist.lpt_shard([sdist.prompt_cost(n) for n in lengths], world)[rank]
    mbs = sdist.micro_batches(shard, lengths, wl["max_tokens"])
    g = torch.Generator().manual_seed(1000 + rank)
    inputs = {}
    for i in shard:
        inputs[i] = (torch.randn(cfg.io_channels, lengths[i], generator=g).to(dev),
                     torch.randn(wl["Tc"], cfg.cond_token_dim, generator=g).to(dev),
                     torch.randn(cfg.global_cond_dim, generator=g).to(dev))
    t = torch.full((max(len(mb) for mb in mbs),), 0.5, device=dev)

    def one_step():
        for mb in mbs:
            xs = [inputs[i][0] for i in mb]
            cond = torch.stack([inputs[i][1] for i in mb])
            gemb = torch.stack([inputs[i][2] for i in mb])
            eng.forward_varlen(xs, t[:len(mb)], cond, gemb, None, cfg_scale=wl["cfg_scale"], apg_scale=wl["apg_scale"])

    with torch.inference_mode():
        for _ in range(args.warmup):
            one_step()
        torch.cuda.synchronize()
        clocks = ClockSampler(local)
        clocks.start()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            one_step()
        e1.record()
        torch.cuda.synchronize()
        barrier(world)
        clk = clocks.stop()
    my_ms = e0.elapsed_time(e1) / args.steps
    ms = max_over_ranks(my_ms, world)
    # per-rank device time and stream rows (latents + memory tokens, both CFG halves): the straggler and the
    # LPT balance the scaling depends on
    rank_ms = gather_over_ranks(my_ms, world)
    rank_rows = gather_over_ranks(float(sum(2 * (lengths[i] + cfg.num_memory_tokens) for i in shard)), world)
    tokens = 2 * sum(lengths)
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": tokens / (ms / 1e3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp8-e4m3 linears / bf16 attention", "data": "synthetic",
            "config": {"workload": args.workload, "model": f"sa3-{wl['model']} DiT, random init",
                       "prompts": wl["n_prompts"], "lengths": f"U{{{wl['len_lo']}..{wl['len_hi']}}} seed 0",
                       "tokens_per_step": tokens, "parallelism": f"dp{world} (LPT, CFG pair per GPU)",
                       "packing": f"variable-length, <= {wl['max_tokens']} rows per batch",
                       "micro_batches_rank0": len(mbs)},
            "per_rank": {"ms": [round(x, 2) for x in rank_ms], "rows": [int(x) for x in rank_rows],
                         "rows_per_s": [round(r / (m / 1e3)) for r, m in zip(rank_rows, rank_ms)]},
            "clocks": clk,
        }), flush=True)


def run_seq_split(args, wl, world, rank, local):
    """One long sequence over all ranks (sa3_b200.seqsplit): per-layer halo exchange, all-reduced APG sums;
    max-over-ranks device time of the whole forward (both CFG halves)."""
    import torch.distributed as dist

    from sa3_b200 import seqsplit as ss
    from sa3_b200.modules import DiffusionTransformer, init_synthetic_

    dev = torch.device("cuda", local)
    cfg = model_cfg(wl["model"])
    eng = init_synthetic_(DiffusionTransformer(cfg), seed=0).quantize(wl["mode"]).engine()
    L = wl["L"]
    sp = ss.make_split(L, rank, world, cfg.num_memory_tokens, cfg.sliding_window,
                       group=dist.group.WORLD if world > 1 else None)
    g = torch.Generator().manual_seed(0)
    x = torch.randn(1, cfg.io_channels, L, generator=g)[..., sp.lat_start:sp.lat_end].to(dev)
    cond = torch.randn(1, wl["Tc"], cfg.cond_token_dim, generator=g).to(dev)
    gemb = torch.randn(1, cfg.global_cond_dim, generator=g).to(dev)
    t = torch.full((1,), 0.5, device=dev)

    def one_step():
        return eng.forward_split(x, t, sp, cond, gemb, None, cfg_scale=wl["cfg_scale"], apg_scale=wl["apg_scale"])

    with torch.inference_mode():
        for _ in range(args.warmup):
            one_step()
        torch.cuda.synchronize()
        clocks = ClockSampler(local)
        clocks.start()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            one_step()
        e1.record()
        torch.cuda.synchronize()
        barrier(world)
        clk = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": 2 * L / (ms / 1e3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp8-e4m3 linears / bf16 attention", "data": "synthetic",
            "config": {"workload": args.workload, "model": f"sa3-{wl['model']} DiT, random init", "L": L,
                       "memory_tokens": cfg.num_memory_tokens, "global_batch": 2,
                       "parallelism": f"sequence split over {world} (halo {cfg.sliding_window})",
                       "tokens_rank0": sp.tok_end - sp.tok_start},
            "clocks": clk,
        }), flush=True)


def run_ours(args, wl, world, rank, local):
    from sa3_b200 import ops, _lib
    from sa3_b200.modules import DiffusionTransformer, init_synthetic_

    dev = torch.device("cuda", local)
    cfg = model_cfg(wl["model"])
    model = init_synthetic_(DiffusionTransformer(cfg), seed=0)
    if wl["mode"] == "gptq":
        from sa3_b200.gptq import random_model_layers
        model.quantize("gptq", gptq_layers=random_model_layers(model, seed=1, device=dev))
    else:
        model.quantize(wl["mode"])
    eng = model.engine()
    x, t, cond, gemb, loc = make_inputs(wl, cfg, seed=100 + rank, device=dev)
    cs, aps = wl["cfg_scale"], wl["apg_scale"]

    # launches per step (one eager step; every C-ABI call is one kernel launch)
    n0 = ops.LAUNCHES
    with torch.inference_mode():
        eng.forward(x, t, cond, gemb, loc, cfg_scale=cs, apg_scale=aps)
    launches_per_step = ops.LAUNCHES - n0
    torch.cuda.synchronize()

    with torch.inference_mode():
        step = eng.graphed(x, t, cond, gemb, loc, cfg_scale=cs, apg_scale=aps)
        for _ in range(args.warmup):
            step(x, t, cond, gemb, loc)
        torch.cuda.synchronize()

        clocks = ClockSampler(local)
        clocks.start()
        time.sleep(0.3)
        barrier(world)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            step.graph.replay()
        e1.record()
        torch.cuda.synchronize()
        barrier(world)
        ms = e0.elapsed_time(e1) / args.steps
        clk = clocks.stop()
    ms_max = max_over_ranks(ms, world)
    tokens_per_gpu = 2 * wl["L"] * wl.get("prompts", 1)
    value = tokens_per_gpu * world / (ms_max / 1e3)

    # ---- e2e: the public module call with pinned HOST inputs (H2D inside), result read back to the host
    model.enable_cuda_graph()
    hx, ht, hc, hg, hl = (a.cpu().pin_memory() for a in (x, t, cond, gemb, loc))
    with torch.inference_mode():
        for _ in range(max(2, args.warmup)):
            model(hx, ht, cross_attn_cond=hc, global_embed=hg, local_add_cond=hl, cfg_scale=cs, apg_scale=aps).cpu()
        torch.cuda.synchronize()
        barrier(world)
        e0.record()
        for _ in range(args.steps):
            v = model(hx, ht, cross_attn_cond=hc, global_embed=hg, local_add_cond=hl, cfg_scale=cs, apg_scale=aps)
            out_host = v.to("cpu")
        e1.record()
        torch.cuda.synchronize()
        barrier(world)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    h2d = sum(a.numel() * a.element_size() for a in (hx, ht, hc, hg, hl))
    d2h = out_host.numel() * out_host.element_size()

    peaks = _peaks()
    bf16_peak, bf16_src = (peaks["bf16_tflops"], "measured bf16 burst (MEASURED_PEAKS.json)") if peaks else \
        (1590.0, "fallback bf16 1.59 PF")
    ws = eng.ws
    reps = 20

    def _timed(fn):
        with torch.inference_mode():
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            e0.record()
            for _ in range(reps):
                fn()
            e1.record()
            torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    # ---- roofline of the dominant kernel: the windowed (differential) self-attention of one block, on the step's
    # own q|k|v rows, timed live with CUDA events on the launching stream (the current stream)
    D, H = cfg.embed_dim, cfg.num_heads
    qkv, o = ws.qkv, ws.o
    wlw, wrw = cfg.sliding_window
    seq = dict(cu_seqlens_q=ws.cu, cu_seqlens_k=ws.cu, max_seqlen_q=ws.max_n, max_seqlen_k=ws.max_n)
    if cfg.differential:
        run_attn = lambda: ops.attention(qkv[:, 0:D], qkv[:, D:2 * D], qkv[:, 2 * D:3 * D], q2=qkv[:, 3 * D:4 * D],  # noqa
                                         k2=qkv[:, 4 * D:5 * D], heads=H, window=(wlw, wrw), out=o, **seq)
    else:
        run_attn = lambda: ops.attention(qkv[:, 0:D], qkv[:, D:2 * D], qkv[:, 2 * D:3 * D], heads=H,  # noqa: E731
                                         window=(wlw, wrw), out=o, **seq)
    a_ms = _timed(run_attn)
    streams = 2 if cfg.differential else 1
    seq_lens = [int(v) for v in (ws.cu_host[1:] - ws.cu_host[:-1])]
    pairs = sum(band_pairs(n, wlw, wrw) for n in seq_lens)
    a_flops = 4.0 * 64 * pairs * H * streams
    a_exps = sum(score_tiles(n, wlw, wrw) for n in seq_lens) * 128 * 128 * H * streams
    sm_count = torch.cuda.get_device_properties(dev).multi_processor_count
    clk_mhz = (clk or {}).get("sm_mhz") or 1965.0
    mufu_floor_ms = a_exps / (16.0 * sm_count * clk_mhz * 1e6) * 1e3  # ex2 at 16 per clock per SM (measured)
    a_ach = a_flops / (a_ms / 1e3) / 1e12
    roofline = {"bound": "tensor", "kernel": "attention_tc_kernel (windowed self-attention, "
                + ("differential, shared V" if cfg.differential else "single stream") + ")",
                "achieved": a_ach, "peak": bf16_peak, "unit": "TFLOP/s", "frac": a_ach / bf16_peak,
                "peak_source": bf16_src + "; bf16 MMA",
                "traffic": _profiled_traffic("attention_diff_swa_medium.md")
                if (cfg.differential and ws.M == 16494) else None,
                "traffic_source": "profiles/attention_diff_swa_medium.md (ncu dram read+write bytes, one launch)",
                "per_launch": {"flops": a_flops, "ms": a_ms, "band_pairs": pairs, "heads": H, "streams": streams,
                               "exp2": a_exps, "mufu_floor_ms": mufu_floor_ms,
                               "mufu_floor_basis": f"16 ex2/clk/SM x {sm_count} SMs at {clk_mhz:.0f} MHz"}}

    # ---- the largest GEMM: the FF GLU.proj with its SwiGLU epilogue, on the step's own buffers
    lin = eng.lin["transformer.layers.0.ff.ff.0.proj"]
    M, K = ws.a.shape
    Nw = lin.n
    if lin.gptq is not None:
        # the path the step takes: the engine picks dequantise-once + bf16 GEMM for many rows
        from sa3_b200.engine import GPTQ_DEQUANT_MIN_ROWS
        run_k = lambda: eng._gemm(ws.a, lin, ws.u, kind=_lib.EPI_SWIGLU)  # noqa: E731
        kname = ("gptq_dequant_orig_kernel + gemm_pair_kernel<bf16, SwiGLU> (FF GLU.proj, int4 weight dequantised "
                 "once per call)" if M >= GPTQ_DEQUANT_MIN_ROWS else
                 "permute_cols_kernel + gemm_gptq_kernel<SwiGLU> (FF GLU.proj, int4 dequant in smem)")
    else:
        scale = ws.scale[4:5]
        run_k = lambda: eng._gemm(ws.a, lin, ws.u, x_scale=scale, kind=_lib.EPI_SWIGLU)  # noqa: E731
        # M >= 512 runs on the 2-SM (CTA pair) kernel, smaller M on the single-SM one
        kern = "gemm_pair_kernel" if M >= 512 else "gemm_persistent_kernel"
        kname = f"{kern}<{'fp8' if lin.fp8 else 'bf16'}, SwiGLU> (FF GLU.proj)"
    k_ms = _timed(run_k)
    flops = 2.0 * M * Nw * K
    achieved = flops / (k_ms / 1e3) / 1e12
    if lin.fp8:
        peak, peak_src = measured_fp8_peak(dev)
        if peak is None:
            peak, peak_src = 2 * bf16_peak, "2x " + bf16_src + " (" + peak_src + ")"
    else:
        peak, peak_src = bf16_peak, bf16_src
    # DRAM bytes of one launch from the committed ncu summary of this exact shape, when there is one
    tprof = ("gemm_fp8_ff1_medium.md" if (lin.fp8 and M == 16494) else
             "gemm_gptq_dense_ff1.md" if (lin.gptq is not None and M == 42368) else None)
    traffic = _profiled_traffic(tprof) if tprof else None
    roofline_gemm = {"bound": "tensor", "kernel": kname, "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "peak_source": peak_src, "traffic": traffic,
                     "traffic_source": f"profiles/{tprof} (ncu dram read+write bytes, one launch)"
                     if traffic else None,
                     "per_launch": {"flops": flops, "ms": k_ms, "M": M, "N": Nw, "K": K}}

    if rank == 0:
        res = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None,
            "dtype": {"fp8": "fp8-e4m3 linears / bf16 attention", "gptq": "int4 weights (GPTQ) / bf16 activations",
                      "bf16": "bf16"}[wl["mode"]],
            "data": "synthetic",
            "config": {"workload": args.workload, "model": f"sa3-{wl['model']} DiT, random init",
                       "dim": cfg.embed_dim, "depth": cfg.depth, "heads": cfg.num_heads,
                       "differential": cfg.differential, "window": list(cfg.sliding_window), "L": wl["L"],
                       "memory_tokens": cfg.num_memory_tokens, "context_tokens": wl["Tc"],
                       "prompts_per_gpu": wl.get("prompts", 1), "global_batch": 2 * wl.get("prompts", 1) * world,
                       "seq_len": wl["L"], "cfg_scale": wl["cfg_scale"], "parallelism": f"dp{world}",
                       "l2": "working set > L2 (1.45 GB FP8 weights + activations per step); no flush"},
            "clocks": clk,
            "e2e": {"value": tokens_per_gpu * world / (e2e_ms / 1e3), "unit": UNIT, "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches_per_step * args.steps,
            "launches_per_step": launches_per_step,
            "roofline": roofline,
            "roofline_gemm": roofline_gemm,
        }
        if world == 1 and not args.no_cpu_baseline:
            threads = len(os.sched_getaffinity(0))
            step_s, meas, n = cpu_dit_sample(wl, threads)
            res["cpu_baseline"] = {"value": tokens_per_gpu / step_s, "unit": UNIT, "cores": threads, "kind": "port",
                                   "sample": _cpu_sample_text(wl, n, meas)}
        print(json.dumps(res), flush=True)
    del step
    model._graphs = None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="medium_fp8")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, wl, world, rank)
        return
    world, rank, local = dist_setup()
    try:
        if wl.get("dp"):
            run_dp_varlen(args, wl, world, rank, local)
        elif wl.get("seq_split"):
            run_seq_split(args, wl, world, rank, local)
        else:
            run_ours(args, wl, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
