#!/usr/bin/env python
"""Benchmark of the B200 engine on BASELINE.json's metric: decode tokens/s of the 110M
Q8_0 model with 64 concurrent requests, plus the paged-attention kernel's achieved HBM
bandwidth.

Workload ("decode64"): 64 requests with uniform-random prompts of U[128, 768] tokens
(seed 100 + rank) are admitted through the reference-mode continuous scheduler
(Continuous_Scheduler::step semantics: one prompt chunk per step, decode of every running
request) until all 64 are running.  A step is then one decode iteration of the whole
batch: 64 tokens, every weight byte and every request's K/V read once per layer.

    value   device-resident: the decode step's kernels re-enqueued from the step
            descriptor already in HBM (nr_replay_decode), K timed steps, CUDA events on the
            engine stream, max over ranks.  Weights (194 MB) + K/V read per step
            (~2.7 GB) exceed the 126 MB L2, so no flush is needed between steps.
    e2e     the public call: nr_step (scheduler + block-table upload from pinned host
            memory + all kernels + greedy tokens copied back), K timed steps.
    roofline  the dominant kernel (paged decode attention): algorithmic bytes per launch
            (sum over rows of ctx * 2 * kv_dim * 4 B of K/V, plus q/out and block tables)
            over its mean launch time from per-launch CUDA events in a second timed pass.
    cpu_baseline  the reference's own forward_decode_batch (oracle/_ref, the ref_fixed
            build) on the host cores, a bounded sample of the same workload.

``--impl reference`` runs only that reference CPU path (rank 0) on the same workload.
Multi-GPU (torchrun): independent replicas, each rank with its own 64 requests (weak
scaling); NCCL is used only for the barrier and the max-over-ranks of the timings."""
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

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from nitrorag_b200 import EngineConfig, NitroEngine, synth  # noqa: E402

METRIC = "decode tok/s per GPU (110M Q8_0, 64 reqs); paged-attn achieved HBM GB/s"
N_REQ = 64
PROMPT_LO, PROMPT_HI = 128, 768
MODEL_SEED = 1234


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "of measured"
    except Exception:
        return 6650.0, "of fallback"


def load_traffic():
    """Per-launch DRAM bytes of the attention kernel from the committed ncu summary,
    scaled by the algorithmic bytes of the captured launch (see profiles/)."""
    path = os.path.join(ROOT, "profiles", "decode_attention_decode64.md")
    try:
        vals = {}
        with open(path) as f:
            for line in f:
                if line.startswith("traffic_ratio:"):
                    vals["ratio"] = float(line.split(":", 1)[1].split()[0])
        return vals.get("ratio")
    except OSError:
        return None


# ------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, ids):
        self.ids = ids
        self.proc = None
        self.out = None

    def start(self):
        try:
            self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", ",".join(str(i) for i in self.ids)], stdout=self.out, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.flush()
        self.out.seek(0)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.out.read().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.out.name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------ workload
def prompts_for(rank: int):
    return synth.decode_workload(N_REQ, PROMPT_LO, PROMPT_HI, 32000, seed=100 + rank)


def schedule_contexts(prompts, extra_steps: int):
    """Context length of every request at the first decode step after all requests are
    running plus `extra_steps` more steps, from a host-only engine replaying the
    reference scheduler (positions do not depend on the sampled token values)."""
    shape = (768, 2048, 12, 12, 12, 32000, 1024)
    eng = NitroEngine(config=EngineConfig(total_blocks=8192, max_new_tokens=100000, device=-1), shape=shape)
    for i, p in enumerate(prompts):
        eng.add_request(i, p)
    while True:
        plan = eng.step_plan()
        eng.step_commit([0] * (int(plan["prefill_done"]) + len(plan["decode_req_ids"])))
        if len(eng.running_batch()) == len(prompts) and plan["prefill_req_id"] < 0:
            break
    for _ in range(extra_steps):
        plan = eng.step_plan()
        eng.step_commit([0] * (int(plan["prefill_done"]) + len(plan["decode_req_ids"])))
    order = eng.running_batch()
    ctx = []
    for rid in order:
        ctx.append(len(prompts[rid]) + len(eng.request_tokens(rid)) - 1)
    eng.close()
    return order, ctx


def attn_bytes(ctx, kv_dim=768, dim=768, B=N_REQ):
    kv = sum(ctx) * 2 * kv_dim * 4
    qo = 2 * B * dim * 4
    bt = sum((c + 15) // 16 for c in ctx) * 4 + B * 4
    return kv + qo + bt


# ------------------------------------------------------------------ CPU reference path
def run_cpu_reference(prompts, ctx_order, ctx, n_steps: int, warmup: int = 0, budget_s: float | None = None):
    """forward_decode_batch of the reference (ref_fixed build) at B=64 with the contexts the
    GPU arm decodes at.  K/V pages are filled with a fixed pattern (decode cost does not
    depend on the values).  Returns (tok/s, threads, steps done, seconds)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    ref = oracle.Reference("fixed")
    threads = os.cpu_count() or 1
    ref.set_threads(threads)
    model = synth.cached_model(synth.SHAPE_110M, seed=MODEL_SEED)
    steps_total = warmup + n_steps
    pages = sum((c + steps_total + 16) // 16 + 1 for c in ctx) + 64
    ref.open(model, N_REQ, pages)
    ref.L.ref_kv_fill(0.5)
    handles = []
    rng = np.random.default_rng(0)
    for rid, c in zip(ctx_order, ctx):
        h = ref.new_request(rid, prompts[rid])
        for t in range(c - 1):
            ref.alloc_token(h, int(rng.integers(0, 32000)))
        handles.append(h)
    toks = [int(rng.integers(0, 32000)) for _ in handles]
    pos = [c - 1 for c in ctx]
    for _ in range(warmup):
        ref.forward_decode(toks, pos, handles)
        pos = [p + 1 for p in pos]
    done = 0
    t0 = time.perf_counter()
    while done < n_steps:
        ref.forward_decode(toks, pos, handles)
        pos = [p + 1 for p in pos]
        done += 1
        if budget_s is not None and time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    ref.close()
    return N_REQ * done / dt, threads, done, dt


def reference_arm(args, rank):
    if rank != 0:
        return 0
    prompts = prompts_for(0)
    order, ctx = schedule_contexts(prompts, args.warmup + args.steps)
    tps, threads, done, dt = run_cpu_reference(prompts, order, ctx, args.steps, warmup=min(args.warmup, 1))
    line = {
        "impl": "reference", "metric": METRIC, "value": round(tps, 3), "unit": "tok/s", "n_gpus": args.gpus,
        "steps": done, "warmup": min(args.warmup, 1), "ms_per_step": round(1000 * dt / max(done, 1), 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(ctx),
        "cpu_baseline": {"value": round(tps, 3), "unit": "tok/s", "cores": threads, "kind": "reference",
                         "sample": f"{done} forward_decode_batch calls at B=64 (ref_fixed build, "
                                   f"{threads} OpenMP threads)"},
        "e2e": {"value": round(tps, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def workload_config(ctx):
    return {"workload": "decode64: one decode step of 64 concurrent requests, 110M Q8_0 "
                        "(dim 768, 12 layers, 12x64 heads, ffn 2048, vocab 32000), paged fp32 KV",
            "model": "llama2-110M-shaped, Q8_0, synthetic N(0,0.02) weights (seed 1234)",
            "batch": N_REQ, "prompt_tokens": f"U[{PROMPT_LO},{PROMPT_HI}]",
            "ctx_mean": round(float(np.mean(ctx)), 1), "ctx_min": int(min(ctx)), "ctx_max": int(max(ctx)),
            "l2": "inputs larger than L2 (194 MB weights + ~2.7 GB K/V read per step)",
            "parallelism": "replicas (one engine per GPU, no collectives)"}


# ------------------------------------------------------------------ GPU arm
def engine_arm(args, rank, world, local_rank):
    import torch
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    torch.cuda.set_device(local_rank)

    def barrier():
        if dist:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if not dist:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    model = synth.cached_model(synth.SHAPE_110M, seed=MODEL_SEED)
    eng = NitroEngine(model, EngineConfig(total_blocks=4096, max_new_tokens=100000, max_batch=N_REQ,
                                          max_prefill_tokens=256, device=local_rank))
    stream = torch.cuda.ExternalStream(eng.stream)
    prompts = prompts_for(rank)
    for i, p in enumerate(prompts):
        eng.add_request(i, p)
    # admission (untimed): until every request is running
    while True:
        r = eng.step()
        if len(eng.running_batch()) == N_REQ and r.prefill_req_id < 0:
            break
    W, K = args.warmup, args.steps

    # ---- e2e: nr_step with host buffers
    for _ in range(W):
        eng.step()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    wall0 = time.perf_counter()
    e0.record(stream)
    for _ in range(K):
        eng.step()
    e1.record(stream)
    torch.cuda.synchronize()
    wall_e2e = time.perf_counter() - wall0
    e2e_ms = max_over_ranks(max(e0.elapsed_time(e1), 1000 * wall_e2e))
    barrier()

    # the state the replays decode at: the last nr_step's batch
    order = eng.running_batch()
    ctx = [len(prompts[rid]) + len(eng.request_tokens(rid)) - 1 for rid in order]

    # ---- value: device-resident replays of that decode step
    eng.replay_decode(W)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ids = [local_rank]
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [int(vis.split(",")[local_rank])]
    sampler = ClockSampler(ids)
    sampler.start()
    time.sleep(0.3)
    launches0 = eng.stats()["kernel_launches"]
    v0, v1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if args.profile_range:  # lets `ncu --profile-from-start off` capture exactly these launches
        torch.cuda.profiler.start()
    v0.record(stream)
    eng.replay_decode(K)
    v1.record(stream)
    torch.cuda.synchronize()
    if args.profile_range:
        torch.cuda.profiler.stop()
    launches = eng.stats()["kernel_launches"] - launches0
    clocks = sampler.stop()
    value_ms = max_over_ranks(v0.elapsed_time(v1))
    barrier()

    # ---- roofline: per-launch events in a second timed pass
    eng.set_profiling(True)
    eng.replay_decode(K)
    kt = eng.kernel_times()
    eng.set_profiling(False)
    attn_ms_total, attn_n = kt["attention"]
    attn_ms = attn_ms_total / max(attn_n, 1)
    peak, peak_src = load_peaks()
    algo = attn_bytes(ctx)
    achieved = algo / (attn_ms * 1e-3) / 1e9
    ratio = load_traffic()
    step_ms_prof = sum(v[0] for v in kt.values()) / K
    kernel_share = {k: round(v[0] / K, 4) for k, v in kt.items()}

    tokens = N_REQ * K * world
    value = tokens / (value_ms * 1e-3)
    e2e = tokens / (e2e_ms * 1e-3)
    h2d = (4 * N_REQ + N_REQ * (1024 // 16)) * 4
    d2h = (N_REQ + 1) * 4

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            p0 = prompts_for(0)
            order0, ctx0 = schedule_contexts(p0, W + K)
            tps, threads, done, dt = run_cpu_reference(p0, order0, ctx0, 100, warmup=1, budget_s=15.0)
            cpu = {"value": round(tps, 3), "unit": "tok/s", "cores": threads, "kind": "reference",
                   "sample": f"{done} forward_decode_batch calls at B=64 ({dt:.1f} s), ref_fixed build of the "
                             f"reference's model_q8.cpp, {threads} OpenMP threads"}
        except Exception as exc:  # the baseline is reported, never required
            cpu = {"value": None, "unit": "tok/s", "cores": None, "kind": "reference",
                   "sample": f"unavailable: {exc}"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": round(value_ms / K, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": workload_config(ctx),
            "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": round(e2e_ms / K, 4)},
            "roofline": {"bound": "hbm", "kernel": "decode_attn_kernel<64>", "achieved": round(achieved, 1),
                         "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4), "peak_source": peak_src,
                         "algorithmic_bytes_per_launch": algo, "launch_ms": round(attn_ms, 5),
                         "traffic": (round(ratio * algo) if ratio else None)},
            "kernel_ms_per_step": kernel_share, "profiled_step_ms": round(step_ms_prof, 4),
            "cpu_baseline": cpu, "clocks": clocks, "gpu_launches": launches,
        }
        print(json.dumps(line), flush=True)
    eng.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["engine", "reference"], default="engine")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-range", action="store_true",
                    help="mark the timed device-resident replays as the CUDA profiler range")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    # contexts grow by one per step; the longest prompt plus admission reaches ~904 of the
    # 1024 positions, so warm-up + timed steps stay within 110
    args.steps = max(1, min(args.steps, 100))
    args.warmup = min(args.warmup, 110 - args.steps)
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        return reference_arm(args, rank)
    return engine_arm(args, rank, world, local_rank)


if __name__ == "__main__":
    sys.exit(main())
