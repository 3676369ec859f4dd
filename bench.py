#!/usr/bin/env python
"""Benchmark of the n-gram speculative-decode hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config llama3-8b]
    python bench.py --impl reference ...      # CPU restatement arm
    python bench.py --config qwen3-4b --kernel-case q4_linear|attention|moe
    python bench.py --kernel-case prefill|prefill_attention|gemm

Default workload (``llama3-8b``): the Llama-3-8B-shape serving configuration,
32 rows per GPU of 4096-token segment-pool prompts; requests arrive Poisson(4)
per verify step and leave after 256 new tokens; n=4, k=4, temperature 0.7,
top-p 0.9, single-draft rejection sampling with per-request seeds
(base seed + request id).  One step is one ``Scheduler.step()``: admission of
waiting requests into free rows (prompt upload, prefill, first token) followed
by one speculative step over the batch (draft -> (k+1)-token verify ->
acceptance + KV rollback).  Weights are random-init N(0, 0.02) quantised to MLX
affine q4 g64 (synthetic; no checkpoint or dataset is read).

The batch starts in steady state: the rows in flight have remaining budgets
spread evenly over 8..256 tokens (the tokens they already generated are part
of their context), so rows finish and waiting requests are admitted at the
steady-state rate inside the timed region.

Rank 0 prints one JSON line.  ``value`` is emitted tokens per second of the
whole job (admission first tokens included) over the CUDA-event device time of
the K steps on the context stream (max over ranks); ``e2e`` is the same metric
on the host clock around the same ``Scheduler.step()`` calls, which upload each
admitted prompt from host memory and copy every step's tokens back to pinned
host memory.  Multi-GPU runs of the dense workloads are request-parallel
replicas (weak scaling, no collective on the data path).
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

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# --------------------------------------------------------------------------- #
# workloads; synthetic inputs with the stated shapes
# --------------------------------------------------------------------------- #
WORKLOADS = {
    "tiny": dict(model="tiny-llama", rows=1, prompt=512, seg_pool=16, seg_len=32, n=3, k=4,
                 temperature=0.0, top_p=0.0, max_new=256,
                 l2="L2-resident (16 MB of q4 weights): latency-bound by design"),
    "qwen3-4b": dict(model="qwen3-4b", rows=8, prompt=2048, seg_pool=64, seg_len=48, n=3, k=5,
                     temperature=0.0, top_p=0.0, max_new=512),
    # the north star's headline: rows join (Poisson, 4 per verify step) and leave mid-flight
    "llama3-8b": dict(model="llama3-8b", rows=32, prompt=4096, seg_pool=64, seg_len=64, n=4, k=4,
                      temperature=0.7, top_p=0.9, max_new=256, arrivals=4.0),
    # the same shapes as a fixed batch (no arrivals): the verify step alone
    "llama3-8b-fixed": dict(model="llama3-8b", rows=32, prompt=4096, seg_pool=64, seg_len=64, n=4, k=4,
                            temperature=0.7, top_p=0.9, max_new=256),
    "qwen3-30b-a3b": dict(model="qwen3-30b-a3b", rows=64, prompt=8192, seg_pool=64, seg_len=64, n=3, k=4,
                          temperature=0.0, top_p=0.0, max_new=256),
    # expert parallel over the run's ranks: the 64 rows split across ranks, experts 128/N per GPU
    "qwen3-30b-a3b-ep": dict(model="qwen3-30b-a3b", rows=64, prompt=8192, seg_pool=64, seg_len=64, n=3, k=4,
                             temperature=0.0, top_p=0.0, max_new=256, ep=True),
    # tensor-parallel over all ranks of the run (does not fit one GPU at 64 rows)
    "llama3-70b": dict(model="llama3-70b", rows=64, prompt=8192, seg_pool=64, seg_len=64, n=4, k=6,
                       temperature=0.0, top_p=0.0, max_new=256, tp=True),
}
DEFAULT_WORKLOAD = "llama3-8b"
WEIGHT_SEED = 20261201
BASE_SEED = 7000          # per-request sampling seed = BASE_SEED + request id
PROMPT_SEED = 910000      # per-request prompt stream seed = PROMPT_SEED + request id
ARRIVAL_SEED = 4242
MIN_CONTEXT = 8
# rows of the CPU restatement's bounded sample (the reference arm and cpu_baseline)
CPU_SAMPLE_ROWS = {"tiny": 1, "qwen3-4b": 8, "llama3-8b": 4, "llama3-8b-fixed": 4, "qwen3-30b-a3b": 4,
                   "qwen3-30b-a3b-ep": 4, "llama3-70b": 1}


def segment_prompt(vocab, n_seg, seg_len, length, seed):
    rng = np.random.default_rng(seed)
    pool = rng.integers(0, vocab, size=(n_seg, seg_len))
    picks = rng.integers(0, n_seg, size=(length + seg_len - 1) // seg_len)
    return pool[picks].reshape(-1)[:length].astype(np.int32)


def model_config(name):
    # engine.py holds only the descriptions; importing it maps no native code
    from mlxcat_b200.engine import CONFIGS
    return CONFIGS[name]


def workload_config(name, wl, world, tp_allreduce="peer"):
    """The `config` object both arms print (identical for the same workload)."""
    tp, ep = bool(wl.get("tp")) and world > 1, bool(wl.get("ep")) and world > 1
    rows = wl["rows"] // world if ep else wl["rows"]
    c = {"workload": name, "model": wl["model"], "rows_per_gpu": rows,
         "global_batch": rows * (1 if tp else world), "prompt_tokens": wl["prompt"],
         "ngram_n": wl["n"], "k": wl["k"], "temperature": wl["temperature"], "top_p": wl["top_p"],
         "max_new_tokens": wl["max_new"],
         "acceptance": ("single-draft rejection sampling, per-request seeds" if wl["temperature"] > 0
                        else "greedy prefix match"),
         "parallelism": (f"tensor-parallel x{world} (" + ("NCCL allreduce" if tp_allreduce == "nccl" else
                                                          "allreduce fused into the row-split projections over "
                                                          "NVLink peer memory") + " per block)" if tp else
                         f"expert-parallel x{world} (NVLink peer-memory exchange per MoE layer)" if ep else
                         f"request-parallel x{world} (replicas, no collective)"),
         "l2": wl.get("l2", "inputs larger than L2 (q4 weights + KV read every step)")}
    if wl.get("arrivals"):
        c["arrivals_per_step"] = wl["arrivals"]
        c["arrival_process"] = "Poisson per verify step; rows leave at max_new_tokens"
    return c


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), "measured"
    return 6650.0, 1400.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        fd, self.path = tempfile.mkstemp(prefix=f"mlxcat_clocks_dev{device}_", suffix=".csv")
        os.close(fd)

    def start(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.fh,
                stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        try:
            os.unlink(self.path)
        except OSError:
            pass
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------------- #
# our arm
# --------------------------------------------------------------------------- #
def reduce_over_ranks(dev_ms, wall, tokens, world, device):
    """Whole-job figures of the timed region: the slowest rank's device and wall
    time (max over ranks) and the tokens of all ranks (sum)."""
    import torch
    if world <= 1:
        return dev_ms, wall, float(tokens)
    t = torch.tensor([dev_ms, wall], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    n = torch.tensor([float(tokens)], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(n, op=torch.distributed.ReduceOp.SUM)
    return float(t[0]), float(t[1]), float(n[0])


def share_tp_id(uid, rank, device):
    """The tensor-parallel group's 128-byte NCCL id, created on rank 0 (uid) and
    broadcast over the job's process group to every rank."""
    import torch
    t = torch.zeros(128, dtype=torch.uint8, device=device)
    if rank == 0:
        t.copy_(torch.frombuffer(bytearray(uid), dtype=torch.uint8))
    torch.distributed.broadcast(t, 0)
    return bytes(t.cpu().numpy().tobytes())


def gather_handles(handle, world, device):
    """Every rank's 128-byte expert-parallel cache handle, in rank order (one
    all-gather over the job's process group)."""
    import torch
    t = torch.frombuffer(bytearray(handle), dtype=torch.uint8).to(device)
    out = [torch.empty_like(t) for _ in range(world)]
    torch.distributed.all_gather(out, t)
    return [bytes(o.cpu().numpy().tobytes()) for o in out]


def job_tokens(tokens, rank, tp):
    """Tokens a rank contributes to the job total: tensor-parallel ranks all
    emit the same rows' tokens, so only rank 0 counts them."""
    return 0 if tp and rank else tokens


def make_request(M, cfg, wl, rank, i, extra=0, max_tokens=None):
    """Request i of a rank's stream: a segment-pool prompt of prompt + extra
    tokens, the workload's sampling with seed BASE_SEED + request id."""
    rid = rank * 1_000_000 + i
    prompt = segment_prompt(cfg.vocab, wl["seg_pool"], wl["seg_len"], wl["prompt"] + extra, PROMPT_SEED + rid)
    sp = M.SamplingParameters(temperature=wl["temperature"], top_p=wl["top_p"], seed=BASE_SEED + rid)
    return M.Request(f"req{rid}", prompt, max_tokens or wl["max_new"], sp)


def arrival_schedule(wl, rank, n_steps, first_id):
    """Seeded Poisson arrivals per step: the request ids that join before each step."""
    rng = np.random.default_rng(ARRIVAL_SEED + rank)
    out, nxt = [], first_id
    for _ in range(n_steps):
        a = int(rng.poisson(wl["arrivals"]))
        out.append(list(range(nxt, nxt + a)))
        nxt += a
    return out


def roofline_of(prof, verify_ms, cfg, rows, k1, lens_before, wbytes, hbm, tflops, peak_kind):
    """Roofline of the dominant kernel class of the verify forward.

    Kernel time per step = (summed CUDA-event time of the class in profiled
    steps, where events bracket every launch) / (the profiled verify forward's
    event time) x the unprofiled, graph-replayed verify forward's device time:
    the class's share of the serialised step applied to the real step."""
    q4_ms = statistics.mean(p["q4_ms"] for p in prof)
    at_ms = statistics.mean(p["attn_ms"] for p in prof)
    pv_ms = statistics.mean(p["verify_ms"] for p in prof)
    q4_share, at_share = q4_ms / pv_ms, at_ms / pv_ms
    q4_t, at_t = q4_share * verify_ms, at_share * verify_ms
    M = rows * k1
    weights = wbytes / 0.5625                      # q4: 0.5 B per weight + 4 B per 64-group
    q4_flops = 2.0 * M * weights
    # K and V bytes per cached token on this rank (a tensor-parallel rank holds n_kv_heads / tp of them)
    kv_tok = 2 * (cfg.n_kv_heads // max(1, cfg.tp_size)) * cfg.head_dim * 2 * cfg.n_layers
    at_bytes = statistics.mean(sum(l + k1 for l in lb) * kv_tok for lb in lens_before)
    tensor_bound = q4_flops / (tflops * 1e12) > wbytes / (hbm * 1e9)
    kern = {
        "q4_linear": {"share_of_verify": q4_share, "ms_per_step": q4_t, "event_ms_serialised": q4_ms,
                      "launches_per_step": prof[0]["q4_n"], "algorithmic_bytes_per_step": wbytes,
                      "flops_per_step": q4_flops, "achieved_gbs": wbytes / (q4_t / 1e3) / 1e9,
                      "achieved_tflops": q4_flops / (q4_t / 1e3) / 1e12},
        "attention": {"share_of_verify": at_share, "ms_per_step": at_t, "event_ms_serialised": at_ms,
                      "launches_per_step": prof[0]["attn_n"], "algorithmic_bytes_per_step": at_bytes,
                      "achieved_gbs": at_bytes / (at_t / 1e3) / 1e9},
    }
    kern["q4_linear"]["frac_hbm"] = kern["q4_linear"]["achieved_gbs"] / hbm
    kern["q4_linear"]["frac_tensor"] = kern["q4_linear"]["achieved_tflops"] / tflops
    kern["attention"]["frac_hbm"] = kern["attention"]["achieved_gbs"] / hbm
    dom = "q4_linear" if q4_t >= at_t else "attention"
    d = kern[dom]
    if dom == "q4_linear" and tensor_bound:
        roof = {"kernel": dom, "bound": "tensor", "achieved": d["achieved_tflops"], "peak": tflops,
                "unit": "TFLOP/s", "frac": d["frac_tensor"],
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json bf16_tflops_sustained; fp16 MMA rate)"}
    else:
        roof = {"kernel": dom, "bound": "hbm", "achieved": d["achieved_gbs"], "peak": hbm, "unit": "GB/s",
                "frac": d["frac_hbm"], "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"}
    roof["kernel_ms_per_step"] = d["ms_per_step"]
    roof["method"] = ("class share of the event-timed (serialised) verify forward x the graph-replayed "
                      "verify forward's device time")
    # DRAM traffic: algorithmic bytes x the DRAM/algorithmic ratio of one ncu capture
    roof["traffic"] = None
    tj = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tj):
        ratios = json.load(open(tj))
        key = cfg.name if cfg.name in ratios else None
        if key and dom in ratios[key]:
            base = wbytes if dom == "q4_linear" else d["algorithmic_bytes_per_step"]
            roof["traffic"] = ratios[key][dom]["ratio"] * base
            roof["traffic_scope"] = ("DRAM bytes per step of the class (algorithmic x the ncu-measured "
                                     "ratio in profiles/traffic.json)")
    return roof, kern


def profiled_steps(cache, do_step, n):
    """n steps with per-launch events; returns each step's class times."""
    out, lens = [], []
    cache.set_profiling(True)
    try:
        do_step()   # capture of the profiled graph (not used)
        for _ in range(n):
            lens.append(cache.lengths())
            do_step()
            q4, at, q4n, atn = cache.profile()
            out.append({"q4_ms": q4, "attn_ms": at, "q4_n": q4n, "attn_n": atn,
                        "verify_ms": cache.last_verify_ms()})
    finally:
        cache.set_profiling(False)
    return out, lens


def run_serving(args, wl, M, A, ctx, cfg, rank, world, local_rank):
    """The Scheduler loop of the arrivals workload (default)."""
    import torch
    rows, k1 = wl["rows"], wl["k"] + 1
    max_len = wl["prompt"] + wl["max_new"] + 16
    spec = M.SpeculativeDecodingConfiguration(True, wl["k"], wl["n"], MIN_CONTEXT, A.ACCEPT_PREFIX)
    sched = M.Scheduler(ctx, rows, max_len, spec, base_seed=BASE_SEED)
    # steady-state start: rows in flight with remaining budgets max_new*(i+1)/rows
    t0 = time.perf_counter()
    for i in range(rows):
        remaining = max(1, wl["max_new"] * (i + 1) // rows)
        sched.submit(make_request(M, cfg, wl, rank, i, extra=wl["max_new"] - remaining, max_tokens=remaining))
    sched.admit_waiting()
    ctx.synchronize()
    setup_s = time.perf_counter() - t0

    n_prof = 2
    total = args.warmup + args.steps + n_prof + 1
    sched_ids = arrival_schedule(wl, rank, total, rows)
    arrivals = [[make_request(M, cfg, wl, rank, i) for i in ids] for ids in sched_ids]
    ext = torch.cuda.ExternalStream(ctx.stream(), device=torch.device("cuda", local_rank))
    cache = sched.generator.cache

    def step(i):
        for r in arrivals[i]:
            sched.submit(r)
        waiting0 = len(sched.waiting)
        out = sched.step()
        admitted = waiting0 - len(sched.waiting)
        return sum(1 for r in out if r.token >= 0), admitted

    for i in range(args.warmup):
        step(i)
    ctx.synchronize()

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        ctx.synchronize()

    clocks = ClockSampler(local_rank)
    if rank == 0:
        clocks.start()
    st0 = sched.speculative_decoding_stats
    launches0 = ctx.launch_count()
    tokens = admitted = 0
    verify = []
    evs = []
    barrier()
    torch.cuda.profiler.start()   # the timed region is the profiler range (ncu --profile-from-start off)
    w0 = time.perf_counter()
    for i in range(args.warmup, args.warmup + args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(ext)
        n, a = step(i)
        e1.record(ext)
        evs.append((e0, e1))
        tokens += n
        admitted += a
        verify.append(cache.last_verify_ms())
    barrier()
    wall = time.perf_counter() - w0
    torch.cuda.profiler.stop()
    clock = clocks.stop() if rank == 0 else None
    launches = ctx.launch_count() - launches0
    st1 = sched.speculative_decoding_stats
    dev_ms = sum(a.elapsed_time(b) for a, b in evs)

    j = [args.warmup + args.steps]

    def prof_step():
        step(j[0])
        j[0] += 1
    prof, lens_before = profiled_steps(cache, prof_step, n_prof)

    dev_ms_max, wall_max, tokens_all = reduce_over_ranks(dev_ms, wall, tokens, world, "cuda")
    if rank:
        return None
    hbm, tflops, peak_kind = peaks()
    roof, kern = roofline_of(prof, statistics.mean(verify), cfg, rows, k1, lens_before,
                             ctx.weights_bytes(), hbm, tflops, peak_kind)
    proposed = st1.proposed_token_count - st0.proposed_token_count
    accepted = st1.accepted_token_count - st0.accepted_token_count
    K = args.steps
    res = {
        "metric": "accepted tok/s", "value": tokens_all / (dev_ms_max / 1e3), "unit": "tok/s",
        "n_gpus": world, "steps": K, "warmup": args.warmup, "ms_per_step": dev_ms_max / K,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded segment-pool prompts, Poisson arrivals, random-init N(0,0.02) q4 weights)",
        "config": workload_config(args.config, wl, world, args.tp_allreduce),
        "verify_step_us": statistics.mean(verify) * 1e3,
        "acceptance_rate": (accepted / proposed if proposed else None),
        "tokens_per_step": tokens / K, "admitted_in_timed_region": admitted,
        "roofline": roof, "kernels": kern,
        "e2e": {"value": tokens_all / wall_max, "unit": "tok/s",
                "h2d_bytes_per_step": (admitted * (wl["prompt"] * 4 + 96)) / K,
                "d2h_bytes_per_step": 4 * (rows * k1 + 2 * rows) + 36 + 4 * admitted / K,
                "api": "Scheduler.step(): mlxcat_cache_insert_row (prompt from host) + mlxcat_spec_step "
                       "(tokens to pinned host)"},
        "gpu_launches": launches, "clocks": clock, "setup_s": setup_s,
    }
    if world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline_from_device(ctx, cache, cfg, wl, spec, args)
    return res


def run_ours(args, wl, rank, world, local_rank):
    import torch
    import mlxcat_b200 as M
    from mlxcat_b200 import _abi as A

    torch.cuda.set_device(local_rank)
    cfg = model_config(wl["model"])
    tp = bool(wl.get("tp")) and world > 1
    ep = bool(wl.get("ep")) and world > 1
    import dataclasses
    if tp:   # every rank runs the same rows on its slice of the model
        cfg = dataclasses.replace(cfg, tp_size=world, tp_rank=rank)
    if ep:   # every rank runs its share of the rows with 1/world of the experts
        cfg = dataclasses.replace(cfg, ep_size=world, ep_rank=rank)
    ctx = M.Context(cfg, local_rank)
    if tp and args.tp_allreduce == "nccl":
        ctx.tp_connect(share_tp_id(M.Context.tp_unique_id() if rank == 0 else None, rank, "cuda"))
    ctx.synth_weights(WEIGHT_SEED, 0.02)
    if wl.get("arrivals"):
        return run_serving(args, wl, M, A, ctx, cfg, rank, world, local_rank)

    prank = 0 if tp else rank   # prompt / seed stream of this rank's rows
    rows, k1 = (wl["rows"] // world if ep else wl["rows"]), wl["k"] + 1
    max_len = wl["prompt"] + wl["max_new"] + 16
    cache = M.BatchKVCache(ctx, rows, max_len)
    if ep or (tp and args.tp_allreduce == "peer"):   # map every rank's exchange region (NVLink peer memory)
        cache.peer_connect(gather_handles(cache.peer_handle(), world, "cuda"))
    spec = M.SpeculativeDecodingConfiguration(True, wl["k"], wl["n"], MIN_CONTEXT, A.ACCEPT_PREFIX)
    t0 = time.perf_counter()
    for r in range(rows):
        req = make_request(M, cfg, wl, prank, r)
        cache.insert_row(r, req.tokens, wl["max_new"], req.sampling)
    ctx.synchronize()
    setup_s = time.perf_counter() - t0

    # budget: rows must not run out of new tokens inside warmup + timed + profiled steps
    budget = (wl["max_new"] - 1) // k1
    n_prof = 2
    if args.warmup + args.steps + n_prof + 1 > budget:
        raise SystemExit(f"--warmup + --steps must be <= {budget - n_prof - 1} for this workload "
                         f"({wl['max_new']} new tokens per row, k={wl['k']})")

    prev_stats = None
    for _ in range(args.warmup):
        prev_stats = cache.spec_step(spec)[3]
    ctx.synchronize()

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        ctx.synchronize()

    # ---- timed region: K steps; device time of each step from the CUDA events
    # the captured step records at its start and end on the context stream ----
    clocks = ClockSampler(local_rank)
    if rank == 0:
        clocks.start()
    launches0 = ctx.launch_count()
    tokens = 0
    last_stats = prev_stats
    barrier()
    torch.cuda.profiler.start()   # the timed region is the profiler range (ncu --profile-from-start off)
    w0 = time.perf_counter()
    dev_ms = 0.0
    verify = []
    for i in range(args.steps):
        tok, n, fin, st = cache.spec_step(spec)
        dev_ms += cache.last_step_ms()
        verify.append(cache.last_verify_ms())
        tokens += int(n.sum())
        last_stats = st
    barrier()
    wall = time.perf_counter() - w0
    torch.cuda.profiler.stop()
    clock = clocks.stop() if rank == 0 else None
    launches = ctx.launch_count() - launches0

    prof, lens_before = profiled_steps(cache, lambda: cache.spec_step(spec), n_prof)

    # ---- aggregate over ranks (tensor parallel: the ranks emit the same tokens) ----
    dev_ms_max, wall_max, tokens_all = reduce_over_ranks(dev_ms, wall, job_tokens(tokens, rank, tp), world,
                                                         "cuda")
    if rank:
        return None
    hbm, tflops, peak_kind = peaks()
    roof, kern = roofline_of(prof, statistics.mean(verify), cfg, rows, k1, lens_before,
                             ctx.weights_bytes(), hbm, tflops, peak_kind)
    proposed = last_stats.proposed_token_count - prev_stats.proposed_token_count
    accepted = last_stats.accepted_token_count - prev_stats.accepted_token_count
    result = {
        "metric": "accepted tok/s", "value": tokens_all / (dev_ms_max / 1e3), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dev_ms_max / args.steps,
        "higher_is_better": True, "scaling": "strong" if tp else "weak", "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic (seeded segment-pool prompts, random-init N(0,0.02) q4 weights)",
        "config": workload_config(args.config, wl, world, args.tp_allreduce),
        "verify_step_us": statistics.mean(verify) * 1e3,
        "acceptance_rate": (accepted / proposed if proposed else None),
        "tokens_per_row_step": tokens / (args.steps * rows),
        "roofline": roof, "kernels": kern,
        "e2e": {"value": tokens_all / wall_max, "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 4 * (rows * k1 + 2 * rows) + 36,
                "api": "mlxcat_spec_step (C ABI, tokens to pinned host memory; no per-step inputs)"},
        "gpu_launches": launches, "launches_before_timed": launches0, "clocks": clock,
        "setup_s": setup_s,
    }
    if world == 1 and not args.no_cpu_baseline and not cfg.n_experts:
        result["cpu_baseline"] = cpu_baseline_from_device(ctx, cache, cfg, wl, spec, args)
    elif cfg.n_experts:
        # copying 17 GB of expert weights into the host restatement is not a
        # bounded sample; the CPU arm for MoE is bench.py --impl reference
        result["cpu_baseline"] = None
    return result


def oracle_config(O, cfg):
    return O.make_config(cfg.n_layers, cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim,
                         cfg.intermediate, cfg.vocab, cfg.tie_embeddings, cfg.qk_norm, cfg.rms_eps,
                         cfg.rope_theta, cfg.n_experts, cfg.top_k, cfg.norm_topk)


def cpu_baseline_from_device(ctx, cache, cfg, wl, spec, args):
    """Time the CPU restatement (oracle) on a bounded sample of the same
    workload: a few of the batch's rows continued from the device's state
    (weights, KV, histories)."""
    from oracle import oracle as O
    from mlxcat_b200 import _abi as A

    cores = O.set_threads(0)
    om = O.Model.empty(oracle_config(O, cfg))
    ids = [A.TENSOR_EMBED] + ([] if cfg.tie_embeddings else [A.TENSOR_LM_HEAD])
    ids += [l * 16 + k for l in range(cfg.n_layers) for k in range(7)]
    shapes = {0: (cfg.n_heads * cfg.head_dim, cfg.hidden), 1: (cfg.n_kv_heads * cfg.head_dim, cfg.hidden),
              2: (cfg.n_kv_heads * cfg.head_dim, cfg.hidden), 3: (cfg.hidden, cfg.n_heads * cfg.head_dim),
              4: (cfg.intermediate, cfg.hidden), 5: (cfg.intermediate, cfg.hidden),
              6: (cfg.hidden, cfg.intermediate)}
    for tid in ids:
        N, K = (cfg.vocab, cfg.hidden) if tid >= A.TENSOR_EMBED else shapes[tid % 16]
        om.set_q4(tid, *ctx.get_q4(tid, N, K))
    active = [r for r, a in enumerate(cache.active()) if a]
    sample = active[:min(len(active), CPU_SAMPLE_ROWS.get(args.config, 2))]
    lens = cache.lengths()
    gen = O.Generator(om, len(sample), cache.max_len,
                      O.SpecConfig(A.ACCEPT_PREFIX, 1, wl["k"], wl["n"], MIN_CONTEXT))
    for i, r in enumerate(sample):
        h = cache.history(r)
        gen.set_row(i, h, 1, wl["max_new"], lens[r],
                    O.sampling(temperature=wl["temperature"], top_p=wl["top_p"], seed=BASE_SEED + r))
        for l in range(cfg.n_layers):
            k16, v16 = cache.extract_row(r, l)
            gen.kv.k(i, l, cfg.n_kv_heads, cfg.head_dim)[:, :lens[r]] = k16.astype(np.float32)
            gen.kv.v(i, l, cfg.n_kv_heads, cfg.head_dim)[:, :lens[r]] = v16.astype(np.float32)
    t0 = time.perf_counter()
    out = gen.step()
    t1 = time.perf_counter() - t0
    n_steps = max(1, min(8, int(20.0 / max(t1, 1e-3))))
    toks = sum(len(o) for o in out)
    t_all = t1
    for _ in range(n_steps - 1):
        t0 = time.perf_counter()
        out = gen.step()
        t_all += time.perf_counter() - t0
        toks += sum(len(o) for o in out)
    return {"value": toks / t_all, "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"{n_steps} speculative steps x {len(sample)} of the batch's rows, continuing from the "
                      f"device state (weights, KV, histories); {t_all:.1f} s of CPU work; admissions "
                      f"(prefill) not included"}


# --------------------------------------------------------------------------- #
# reference arm: the CPU restatement of mlxcat's path, on the host cores
# --------------------------------------------------------------------------- #
def run_reference(args, wl, world):
    from oracle import oracle as O
    cfg = model_config(wl["model"])
    cores = O.set_threads(0)   # every host core, whatever OMP_NUM_THREADS torchrun set
    t0 = time.perf_counter()
    om = O.Model.synth(oracle_config(O, cfg), WEIGHT_SEED, 0.02)
    synth_s = time.perf_counter() - t0
    rows, k1 = CPU_SAMPLE_ROWS.get(args.config, 2), wl["k"] + 1
    max_len = wl["prompt"] + wl["max_new"] + 16
    gen = O.Generator(om, rows, max_len, O.SpecConfig(O.MODE_PREFIX, 1, wl["k"], wl["n"], MIN_CONTEXT))
    # The prompt KV is left at zeros instead of a full-prompt CPU prefill per row
    # (a 4096-token prefill of the 8B model is ~65 TFLOP on the host).  Attention
    # still reads every cached position, so the per-step cost is exact.
    for r in range(rows):
        p = segment_prompt(cfg.vocab, wl["seg_pool"], wl["seg_len"], wl["prompt"], PROMPT_SEED + r).tolist()
        sp = O.sampling(temperature=wl["temperature"], top_p=wl["top_p"], seed=BASE_SEED + r)
        lg = O.forward(om, gen.kv, [p[-1]], [r], [len(p) - 1])[0]
        gen.set_row(r, p + [int(np.argmax(lg))], 1, wl["max_new"], len(p), sp)
    budget = (wl["max_new"] - 1) // k1
    t0 = time.perf_counter()
    gen.step()
    t1 = time.perf_counter() - t0
    # bounded sample: about a minute of timed steps
    steps = max(1, min(args.steps, budget - 1, int(60.0 / max(t1, 1e-3))))
    warm = min(max(0, args.warmup - 1), max(0, budget - 1 - steps))
    for _ in range(warm):
        gen.step()
    toks = 0
    t0 = time.perf_counter()
    for _ in range(steps):
        out = gen.step()
        toks += sum(len(o) for o in out)
    dt = time.perf_counter() - t0
    value = toks / dt
    return {"metric": "accepted tok/s", "value": value, "unit": "tok/s", "impl": "reference",
            "n_gpus": 0, "steps": steps, "warmup": warm + 1, "ms_per_step": dt / steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded segment-pool prompts, random-init N(0,0.02) q4 weights)",
            "config": workload_config(args.config, wl, world, args.tp_allreduce),
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": "port",
                             "sample": f"{steps} speculative steps x {rows} rows of the workload "
                                       f"(weights synthesised on the host in {synth_s:.0f} s, prompt KV "
                                       f"zero-filled, no arrivals or prefill)"},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "mlxcat is Swift/MLX (no toolchain here); the arm times the C restatement of its path "
                    "(oracle/) on every host thread"}


# --------------------------------------------------------------------------- #
# single-kernel cases (isolated roofline timing and small ncu captures)
# --------------------------------------------------------------------------- #
def run_kernel_case(args):
    """Repeated launches of one hot kernel at the workload's verify shape
    through the operator ABI, cycling over enough distinct operands that each
    launch reads cold from HBM (operands > L2).  Prints one JSON line with the
    CUDA-event time per launch and the achieved algorithmic GB/s."""
    import ctypes as C
    import torch
    from mlxcat_b200 import _abi as A

    L = A.lib()
    wl = WORKLOADS[args.config]
    cfg = model_config(wl["model"])
    rows, k1 = wl["rows"], wl["k"] + 1
    M = rows * k1
    hbm, _, peak_kind = peaks()
    torch.cuda.set_device(0)
    p = lambda t: C.c_void_p(t.data_ptr())
    reps = args.kernel_reps
    if args.kernel_case == "prefill":
        run_prefill_case(args, wl, cfg)
        return
    if args.kernel_case == "prefill_attention":
        # the admission's causal attention over one 4096-token prompt chunk
        # (mlxcat_op_prefill_attention, one layer); a few tens of MB on the device
        n, Hq, Hkv, D = 4096, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        q = (torch.randn((n, Hq * D), device="cuda") * 0.5).half()
        kc = (torch.randn((1, Hkv, n, D), device="cuda") * 0.5).half()
        vc = torch.randn((1, Hkv, n, D), device="cuda").half()
        out = torch.empty((n, Hq * D), dtype=torch.float16, device="cuda")
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        flops = 4.0 * Hq * D * n * (n + 1) / 2

        def launch():
            A.check(L.mlxcat_op_prefill_attention(p(q), p(kc), p(vc), 1, n, 0, 0, n, Hq, Hkv, D, p(out), p(err),
                                                  None))
        for i in range(args.warmup):
            launch()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(reps):
            launch()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        print(json.dumps({"kernel_case": "prefill_attention", "config": args.config,
                          "shape": {"tokens": n, "Hq": Hq, "Hkv": Hkv, "D": D, "causal": True},
                          "us_per_launch": ms * 1e3, "tflops": flops / (ms / 1e3) / 1e12,
                          "timeout_flag": int(err.item())}))
        return
    if args.kernel_case == "gemm":
        # the prefill's fused gate/up GEMM on one 2048-token chunk (fp16 weights, tcgen05)
        N, K, Mt = 2 * cfg.intermediate, cfg.hidden, 2048
        w = (torch.randn((N, K), device="cuda") * 0.02).half()
        x = torch.randn((Mt, K), device="cuda").half()
        out = torch.empty((Mt, N // 2), dtype=torch.float16, device="cuda")
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        flops = 2.0 * Mt * N * K

        def launch(i):
            A.check(L.mlxcat_op_gemm_f16(p(w), N, K, p(x), Mt, A.GEMM_SWIGLU, p(out), N // 2, p(err), None))
        for i in range(args.warmup):
            launch(i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(reps):
            launch(i)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        _, tfl, _ = peaks()
        burst = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["bf16_tflops"] \
            if os.path.exists(os.path.join(ROOT, "MEASURED_PEAKS.json")) else 1590.0
        print(json.dumps({"kernel_case": "gemm", "config": args.config,
                          "shape": {"M": Mt, "N": N, "K": K, "epilogue": "swiglu"}, "us_per_launch": ms * 1e3,
                          "tflops": flops / (ms / 1e3) / 1e12, "frac_of_burst_bf16": flops / (ms / 1e3) / 1e12 / burst,
                          "timeout_flag": int(err.item())}))
        return
    if args.kernel_case == "q4_linear":
        N, K = 2 * cfg.intermediate, cfg.hidden          # fused gate/up projection
        copies = max(2, int(4 * 126e6 // (N * K // 2)) + 1)
        W = [torch.randint(-2**31, 2**31 - 1, (N, K // 8), dtype=torch.int32, device="cuda")
             for _ in range(copies)]
        S = [(torch.rand((N, K // 64), device="cuda") * 1e-2).half() for _ in range(copies)]
        B = [(torch.rand((N, K // 64), device="cuda") * -1e-2).half() for _ in range(copies)]
        x = torch.randn((M, K), device="cuda").half()
        ws_bytes = L.mlxcat_op_q4_linear_workspace(N, K, M)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
        y = torch.empty((M, N), dtype=torch.float32, device="cuda")
        algo = N * K // 2 + N * (K // 64) * 4 + M * K * 2 + M * N * 4

        def launch(i):
            j = i % copies
            A.check(L.mlxcat_op_q4_linear(p(W[j]), p(S[j]), p(B[j]), N, K, p(x), M, p(y), p(ws),
                                          ws_bytes, None))
        shape = {"N": N, "K": K, "M": M, "copies": copies}
    elif args.kernel_case == "moe":
        # one layer's sparse MoE MLP (router, gate/up + SwiGLU, down, combine);
        # the experts of one layer (E x 3 q4 matrices) are larger than L2
        H, I, E, TK = cfg.hidden, cfg.intermediate, cfg.n_experts, cfg.top_k
        if not E:
            raise SystemExit("--kernel-case moe needs a MoE workload")
        copies = 2
        shapes = ((I, H), (I, H), (H, I))
        Wt = [[(torch.randint(-2**31, 2**31 - 1, (E, n, k // 8), dtype=torch.int32, device="cuda"),
                (torch.rand((E, n, k // 64), device="cuda") * 1e-2).half(),
                (torch.rand((E, n, k // 64), device="cuda") * -1e-2).half()) for (n, k) in shapes]
              for _ in range(copies)]
        router = (torch.randn((E, H), device="cuda") * 0.02).to(torch.bfloat16)
        x = torch.randn((M, H), device="cuda").half()
        y = torch.empty((M, H), dtype=torch.float32, device="cuda")
        ws_bytes = L.mlxcat_op_moe_workspace(M, H, I, E, TK)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
        ptrs = [tuple(A._vp3(*[Wt[j][kind][f].data_ptr() for kind in range(3)]) for f in range(3))
                for j in range(copies)]
        algo = E * 3 * (I * H // 2 + I * (H // 64) * 4) + E * H * 2 + M * H * 2 + M * H * 4

        def launch(i):
            wq, sc, bi = ptrs[i % copies]
            A.check(L.mlxcat_op_moe(p(x), M, H, I, E, TK, 1, p(router), wq, sc, bi, p(y), None, None,
                                    p(ws), ws_bytes, None))
        shape = {"M": M, "hidden": H, "intermediate": I, "experts": E, "top_k": TK, "copies": copies}
    else:
        Hq, Hkv, D = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        ctx_len = wl["prompt"] + wl["max_new"] // 2
        max_len = ctx_len + k1 + 8
        layers = max(2, int(4 * 126e6 // (2 * rows * Hkv * max_len * D * 2)) + 1)
        kc = [torch.randn((rows, Hkv, max_len, D), device="cuda").half() for _ in range(layers)]
        vc = [torch.randn((rows, Hkv, max_len, D), device="cuda").half() for _ in range(layers)]
        q = torch.randn((M, Hq, D), device="cuda").half()
        trow = torch.arange(rows, dtype=torch.int32, device="cuda").repeat_interleave(k1)
        tpos = (ctx_len + torch.arange(k1, dtype=torch.int32, device="cuda")).repeat(rows)
        out = torch.empty((M, Hq * D), dtype=torch.float16, device="cuda")
        ws_bytes = L.mlxcat_op_attention_workspace(M, k1, Hq, Hkv, D, max_len)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
        algo = 2 * rows * Hkv * (ctx_len + k1) * D * 2 + M * Hq * D * 4

        def launch(i):
            j = i % layers
            A.check(L.mlxcat_op_attention(p(q), p(kc[j]), p(vc[j]), max_len, p(trow), p(tpos), M, k1,
                                          Hq, Hkv, D, p(out), p(ws), ws_bytes, None))
        shape = {"rows": rows, "k1": k1, "ctx": ctx_len, "Hq": Hq, "Hkv": Hkv, "D": D, "layers": layers}
    for i in range(args.warmup):
        launch(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(reps):
        launch(args.warmup + i)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    gbs = algo / (ms / 1e3) / 1e9
    print(json.dumps({"kernel_case": args.kernel_case, "config": args.config, "shape": shape,
                      "us_per_launch": ms * 1e3, "algorithmic_bytes": algo, "achieved_gbs": gbs,
                      "peak_gbs": hbm, "frac": gbs / hbm, "peak_source": peak_kind,
                      "note": "time per launch includes the split-K reduction / combine kernel"}))


def run_prefill_case(args, wl, cfg):
    """Admission of one 4096-token prompt (prefill of every position + the
    first token) on an otherwise idle batch, timed with CUDA events on the
    context stream; flops = 2 x weights x tokens + causal attention."""
    import torch
    import mlxcat_b200 as M
    from mlxcat_b200 import _abi as A
    ctx = M.Context(cfg, 0)
    ctx.synth_weights(WEIGHT_SEED, 0.02)
    n = wl["prompt"]
    cache = M.BatchKVCache(ctx, 2, n + 64)
    ext = torch.cuda.ExternalStream(ctx.stream(), device=torch.device("cuda", 0))
    times = []
    for i in range(args.warmup + args.kernel_reps):
        req = make_request(M, cfg, wl, 0, i)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(ext)
        cache.insert_row(i % 2, req.tokens, 8, req.sampling)
        e1.record(ext)
        torch.cuda.synchronize()
        if i >= args.warmup:
            times.append(e0.elapsed_time(e1))
        cache.remove_row(i % 2)
    ms = statistics.median(times)
    weights = ctx.weights_bytes() / 0.5625
    head = cfg.vocab * cfg.hidden
    lin_flops = 2.0 * (weights - head) * n + 2.0 * head
    att_flops = 4.0 * cfg.n_layers * cfg.n_heads * cfg.head_dim * n * (n + 1) / 2
    print(json.dumps({"kernel_case": "prefill", "config": args.config, "prompt_tokens": n,
                      "ms_per_admission": ms, "ms_all": times, "tokens_per_s": n / (ms / 1e3),
                      "linear_tflop": lin_flops / 1e12, "attention_tflop": att_flops / 1e12,
                      "tflops": (lin_flops + att_flops) / (ms / 1e3) / 1e12}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default=DEFAULT_WORKLOAD, choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="mlxcat", choices=["mlxcat", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--kernel-case", choices=["q4_linear", "attention", "moe", "gemm", "prefill",
                                              "prefill_attention"])
    ap.add_argument("--kernel-reps", type=int, default=50)
    ap.add_argument("--tp-allreduce", default="peer", choices=["peer", "nccl"],
                    help="tensor-parallel allreduce: fused over peer memory, or one NCCL call per block")
    args = ap.parse_args()
    if args.kernel_case:
        run_kernel_case(args)
        return
    if args.warmup < 3 and args.impl == "mlxcat":
        raise SystemExit("--warmup must be >= 3")
    wl = WORKLOADS[args.config]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        # the CPU arm runs once, on rank 0; the other ranks have no work
        if rank == 0:
            print(json.dumps(run_reference(args, wl, world)), flush=True)
        return

    if world > 1:
        import datetime
        import torch
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local_rank))
    res = run_ours(args, wl, rank, world, local_rank)
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
