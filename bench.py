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


# A decoder as narrow as the reference harness allows with the 110M model's vocabulary,
# sequence length and scheduler budget: its Continuous_Scheduler admits and decodes the
# decode64 requests in the same steps as the 110M model (admission and positions are
# count-driven, src/pagedMemory.hpp:317-398), in seconds on the CPU.
SCHED_SHAPE = synth.ModelShape(32, 64, 1, 1, 1, 32000, 1024)


def schedule_contexts(prompts, extra_steps: int):
    """Context length of every request (in running-batch order) at the first decode step
    after all requests are running plus `extra_steps` more steps, from the reference's own
    Continuous_Scheduler::step (oracle/_ref, ref_fixed build) on SCHED_SHAPE: one prompt
    chunk of at most 256 tokens per step, every running request decoded per step."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    ref = oracle.Reference("fixed")
    ref.set_threads(os.cpu_count() or 1)
    pages = sum((len(p) + extra_steps + 300) // 16 + 2 for p in prompts) + 64
    ref.open(synth.cached_model(SCHED_SHAPE, seed=MODEL_SEED), 256, pages)
    ref.sched_reset()
    handles = []
    for i, p in enumerate(prompts):
        h = ref.new_request(i, p)
        ref.sched_add(h)
        handles.append(h)
    for _ in range(4 * len(prompts) + 64):
        before = ref.L.ref_sched_waiting()
        ref.sched_step(100000)
        if before == 0 and len(ref.sched_running()) == len(prompts) and all(
                ref.req_flags(h)["is_prefill_done"] for h in handles):
            break
    else:
        raise RuntimeError("reference scheduler did not admit every request")
    for _ in range(extra_steps):
        ref.sched_step(100000)
    order = ref.sched_running()
    ctx = [len(prompts[rid]) + len(ref.generated(handles[rid])) - 1 for rid in order]
    ref.close()
    return order, ctx


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


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
    """The reference's own CPU path (oracle/_ref only: its scheduler for the contexts, its
    forward_decode_batch for the timed steps); no library of this repository is loaded."""
    if rank != 0:
        return 0
    prompts = prompts_for(0)
    order, ctx = schedule_contexts(prompts, args.warmup + args.steps)
    tps, threads, done, dt = run_cpu_reference(prompts, order, ctx, args.steps, warmup=args.warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(tps, 3), "unit": "tok/s", "n_gpus": args.gpus,
        "steps": done, "warmup": args.warmup, "ms_per_step": round(1000 * dt / max(done, 1), 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(ctx),
        "cpu_baseline": {"value": round(tps, 3), "unit": "tok/s", "cores": threads, "kind": "reference",
                         "cpu_model": cpu_model(),
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


# ------------------------------------------------------------------ other configs
# The survey's other workloads, one JSON line each (`--workload config1|config3|config4|
# config5`); the default `decode64` line above is the headline.  All run on one GPU.
W110_BYTES = 193_932_288          # Q8 projections + fp32 classifier + RMS gains, 110M
KV110_PER_TOKEN = 12 * 2 * 768 * 4  # K and V of every layer, 110M


def _dev_events(torch, stream):
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def _profile_classes(eng, n):
    eng.set_profiling(True)
    eng.replay_decode(n)
    kt = eng.kernel_times()
    eng.set_profiling(False)
    return {k: (v[0] / n, v[1] // max(n, 1)) for k, v in kt.items()}


def run_config1(args):
    """Config 1: one request, 256-token prompt, 128 greedy tokens (B = 1 decode: the Q8_0
    matvec path).  value = device-resident decode step at the end of the run;
    e2e = the 127 decode steps through nr_step."""
    import torch
    peak, peak_src = load_peaks()
    model = synth.cached_model(synth.SHAPE_110M, seed=MODEL_SEED)
    eng = NitroEngine(model, EngineConfig(total_blocks=64, max_new_tokens=128, max_batch=1, max_prefill_tokens=256,
                                          device=0))
    stream = torch.cuda.ExternalStream(eng.stream)
    prompt = np.random.default_rng(11).integers(0, 32000, 256).astype(np.int32)
    eng.add_request(0, prompt)
    t0 = time.perf_counter()
    eng.step()  # prefill of the whole prompt (budget 256) and the first token
    prefill_s = time.perf_counter() - t0
    t0 = time.perf_counter()
    n_dec = 0
    while eng.has_active_requests():
        r = eng.step()
        n_dec += r.n_decode
    e2e_s = time.perf_counter() - t0
    pos = 256 + 127 - 1  # position of the last decode step (replayed below)
    eng.replay_decode(args.warmup)
    torch.cuda.synchronize()
    e0, e1 = _dev_events(torch, stream)
    e0.record(stream)
    eng.replay_decode(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    step_ms = e0.elapsed_time(e1) / args.steps
    step_bytes = W110_BYTES + (pos + 1) * KV110_PER_TOKEN + KV110_PER_TOKEN
    prof = _profile_classes(eng, args.steps)
    per_class_bytes = {"qkv": 12 * 2304 * 768 * 1.125, "wo": 12 * 768 * 768 * 1.125, "w13": 12 * 4096 * 768 * 1.125,
                       "w2": 12 * 768 * 2048 * 1.125, "logits": 32000 * 768 * 4,
                       "attention": (pos + 1) * KV110_PER_TOKEN}
    kernels = {}
    for k, nb in per_class_bytes.items():
        ms = prof[k][0]
        kernels[k] = {"ms_per_step": round(ms, 4), "GB/s": round(nb / (ms * 1e-3) / 1e9, 1),
                      "frac": round(nb / (ms * 1e-3) / 1e9 / peak, 3)}
    matvec_bytes = sum(per_class_bytes[k] for k in ("qkv", "wo", "w13", "w2", "logits"))
    matvec_ms = sum(prof[k][0] for k in ("qkv", "wo", "w13", "w2", "logits"))
    eng.close()
    return {"workload": "config1", "metric": "decode tok/s, 1 request (110M Q8_0, 256-token prompt, 128 greedy tokens)",
            "value": round(1000.0 / step_ms, 1), "unit": "tok/s", "ms_per_step": round(step_ms, 4),
            "e2e": {"value": round(n_dec / e2e_s, 1), "unit": "tok/s", "decode_steps": n_dec},
            "prefill_ms": round(1000 * prefill_s, 3),
            "roofline": {"bound": "hbm", "bytes_per_step": step_bytes,
                         "achieved": round(step_bytes / (step_ms * 1e-3) / 1e9, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(step_bytes / (step_ms * 1e-3) / 1e9 / peak, 4), "peak_source": peak_src},
            "matvec": {"bytes_per_step": int(matvec_bytes), "ms_per_step": round(matvec_ms, 4),
                       "achieved": round(matvec_bytes / (matvec_ms * 1e-3) / 1e9, 1),
                       "frac": round(matvec_bytes / (matvec_ms * 1e-3) / 1e9 / peak, 4),
                       "note": "per-launch CUDA events around every matvec launch (second pass)"},
            "kernels": kernels, "steps": args.steps}


def run_config3(args):
    """Config 3: 50 requests arriving by a seeded Poisson process (mean 20 req/s), prompts
    U[64, 512], 60 % of them sharing a 384-token prefix, 256 greedy tokens each, through
    nr_step (reference scheduler, prefix cache on).  Arrivals are mapped to steps by a
    virtual clock (step k admits every arrival <= k x 10 ms), so the admission sequence is
    deterministic; value = generated tokens over the wall time of the whole run."""
    rng = np.random.default_rng(33)
    arrive = np.cumsum(rng.exponential(1 / 20.0, 50))
    shared = rng.integers(0, 32000, 384).astype(np.int32)
    prompts = []
    for _ in range(50):
        if rng.random() < 0.6:
            n = int(rng.integers(385, 513))
            prompts.append(np.concatenate([shared, rng.integers(0, 32000, n - 384).astype(np.int32)]))
        else:
            prompts.append(rng.integers(0, 32000, int(rng.integers(64, 513))).astype(np.int32))
    model = synth.cached_model(synth.SHAPE_110M, seed=MODEL_SEED)
    eng = NitroEngine(model, EngineConfig(total_blocks=4096, max_new_tokens=256, max_batch=64, max_prefill_tokens=256,
                                          device=0))
    dt = 0.010
    k, nxt, gen, hits, steps = 0, 0, 0, 0, 0
    t0 = time.perf_counter()
    while nxt < 50 or eng.has_active_requests():
        while nxt < 50 and arrive[nxt] <= k * dt:
            eng.add_request(nxt, prompts[nxt])
            nxt += 1
        if eng.has_active_requests():
            r = eng.step()
            gen += len(r.emitted)
            hits += r.prefill_hits
            steps += 1
        k += 1
    wall = time.perf_counter() - t0
    st = eng.stats()
    eng.close()
    return {"workload": "config3", "metric": "aggregate tok/s, 50 Poisson requests with a shared prefix (110M Q8_0)",
            "value": round(gen / wall, 1), "unit": "tok/s", "generated_tokens": gen, "wall_s": round(wall, 3),
            "steps": steps, "prefix_hit_pages": hits, "evictions": st["evictions"],
            "note": "virtual clock 10 ms per step for admission; wall time includes the scheduler and copies"}


def _config4_packed(model, prompts):
    """The same 32 prompts through nr_step in NR_SCHED_PACKED with a 4096-token budget:
    four 1024-token prompts per step in one forward pass (max_new_tokens 1, so every step
    is pure prefill: the four finish and are released at the next step)."""
    import torch
    from nitrorag_b200 import NR_SCHED_PACKED
    eng = NitroEngine(model, EngineConfig(total_blocks=36 * 66, max_new_tokens=1, max_batch=32,
                                          max_tokens_per_batch=4096, max_prefill_tokens=4096, device=0,
                                          sched_mode=NR_SCHED_PACKED))
    stream = torch.cuda.ExternalStream(eng.stream)
    # warm-up round (kernel set-up, one packed step) on other prompts: the timed prompts
    # must not find their pages in the prefix cache
    warm = np.random.default_rng(45).integers(0, 32000, (4, 1024)).astype(np.int32)
    for i in range(4):
        eng.add_request(1000 + i, warm[i])
    while eng.has_active_requests():
        eng.step()
    for i, p in enumerate(prompts):
        eng.add_request(i, p)
    torch.cuda.synchronize()
    e0, e1 = _dev_events(torch, stream)
    t0 = time.perf_counter()
    e0.record(stream)
    steps = chunks = 0
    while eng.has_active_requests():
        r = eng.step()
        steps += 1
        chunks += r.n_prefill
    e1.record(stream)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    ms = e0.elapsed_time(e1)
    eng.close()
    return {"value": round(32768 / (ms * 1e-3), 1), "unit": "tok/s", "prefill_ms": round(ms, 3),
            "wall_ms": round(1000 * wall, 3), "steps": steps, "chunks": chunks, "budget": 4096}


def run_config4(args):
    """Config 4: 32 prompts of 1024 tokens prefilled (one 1024-token chunk each through
    nr_forward_prefill), then 16 decode steps at B = 32.  Positions reach 1039, so the
    model header has seq_len 2048."""
    import torch
    model = synth.cached_model(synth.SHAPE_110M_LONG, seed=MODEL_SEED)
    eng = NitroEngine(model, EngineConfig(total_blocks=36 * 66, max_new_tokens=100000, max_batch=32,
                                          max_prefill_tokens=1024, device=0))
    stream = torch.cuda.ExternalStream(eng.stream)
    rng = np.random.default_rng(44)
    prompts = [rng.integers(0, 32000, 1024).astype(np.int32) for _ in range(32)]
    warm = eng.seq_create(1000)
    eng.forward_prefill_chunk(warm, prompts[0], 0, want_logits=False)
    eng.release(warm)
    seqs = [eng.seq_create(i) for i in range(32)]
    torch.cuda.synchronize()
    e0, e1 = _dev_events(torch, stream)
    t0 = time.perf_counter()
    e0.record(stream)
    toks = []
    for s, p in zip(seqs, prompts):
        toks.append(eng.forward_prefill_chunk(s, p, 0, want_logits=False)[1])
    e1.record(stream)
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0
    prefill_dev_ms = e0.elapsed_time(e1)
    # per-kernel-class breakdown of one more prefill (CUDA events around every launch)
    extra = eng.seq_create(2000)
    eng.set_profiling(True)
    eng.forward_prefill_chunk(extra, prompts[1], 0, want_logits=False)
    kt = eng.kernel_times()
    eng.set_profiling(False)
    eng.release(extra)
    pos = [1024] * 32
    t0 = time.perf_counter()
    for _ in range(16):
        _, am = eng.forward_decode_batch(toks, pos, seqs, want_logits=False)
        toks = am.tolist()
        pos = [p + 1 for p in pos]
    decode_s = time.perf_counter() - t0
    eng.close()
    packed = _config4_packed(model, prompts)
    linear = 2 * 84_934_656 * 32768
    attn = 2 * 2 * 12 * 64 * 12 * 32 * (1024 * 1025 // 2)
    flops = linear + attn
    _, peak_src = load_peaks()
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            tf_peak = float(json.load(f)["bf16_tflops"])
    except Exception:
        tf_peak = 1590.0
    tflops = flops / (prefill_dev_ms * 1e-3) / 1e12
    issued = 3 * (linear + attn) / (prefill_dev_ms * 1e-3) / 1e12  # tensor work incl. the hi/lo split
    return {"workload": "config4", "metric": "prefill tok/s, 32 x 1024-token prompts (110M Q8_0)",
            "value": round(32768 / (prefill_dev_ms * 1e-3), 1), "unit": "tok/s",
            "prefill_ms": round(prefill_dev_ms, 3), "prefill_wall_ms": round(1000 * prefill_s, 3),
            "model_tflops": round(tflops, 2),
            "roofline": {"bound": "tensor", "achieved": round(issued, 2), "peak": tf_peak, "unit": "TFLOP/s",
                         "frac": round(issued / tf_peak, 4), "peak_source": peak_src,
                         "note": "bf16 tensor FLOPs issued: 3 x (linear + causal attention), the hi/lo split"},
            "decode_b32": {"value": round(32 * 16 / decode_s, 1), "unit": "tok/s", "steps": 16},
            "packed_scheduler": packed,
            "prefill_kernel_ms_per_prompt": {k: round(v[0], 3) for k, v in kt.items()}}


def run_config5(args):
    """Config 5 (reduced): the 7B-shaped model, B requests (default 64) with 512-token
    prompts prefilled one per call, then 32 decode steps at batch B through
    nr_forward_decode.  The full 256-request run needs ~160 GiB of K/V on one GPU."""
    import torch
    B = args.batch or 64
    t0 = time.perf_counter()
    model = synth.cached_model_on_device(synth.SHAPE_7B, seed=MODEL_SEED)  # 7.8 GB, values from torch's RNG
    gen_s = time.perf_counter() - t0
    pages = B * (512 // 16 + 4) + 16
    eng = NitroEngine(model, EngineConfig(total_blocks=pages, max_new_tokens=100000, max_batch=B,
                                          max_prefill_tokens=512, device=0))
    stream = torch.cuda.ExternalStream(eng.stream)
    rng = np.random.default_rng(55)
    prompts = [rng.integers(0, 32000, 512).astype(np.int32) for _ in range(B)]
    seqs = [eng.seq_create(i) for i in range(B)]
    torch.cuda.synchronize()
    e0, e1 = _dev_events(torch, stream)
    e0.record(stream)
    toks = [eng.forward_prefill_chunk(s, p, 0, want_logits=False)[1] for s, p in zip(seqs, prompts)]
    e1.record(stream)
    torch.cuda.synchronize()
    prefill_ms = e0.elapsed_time(e1)
    pos = [512] * B
    for _ in range(2):
        _, am = eng.forward_decode_batch(toks, pos, seqs, want_logits=False)
        toks = am.tolist()
        pos = [p + 1 for p in pos]
    n = 30
    t0 = time.perf_counter()
    for _ in range(n):
        _, am = eng.forward_decode_batch(toks, pos, seqs, want_logits=False)
        toks = am.tolist()
        pos = [p + 1 for p in pos]
    dec_s = time.perf_counter() - t0
    eng.replay_decode(3)
    torch.cuda.synchronize()
    d0, d1 = _dev_events(torch, stream)
    d0.record(stream)
    eng.replay_decode(10)
    d1.record(stream)
    torch.cuda.synchronize()
    step_ms = d0.elapsed_time(d1) / 10
    prof = _profile_classes(eng, 3)
    eng.close()
    w_bytes = 7_810_859_008
    kv = sum(p + 1 for p in pos) * 32 * 2 * 4096 * 4
    peak, peak_src = load_peaks()
    return {"workload": "config5", "metric": f"decode tok/s, 7B-shaped Q8_0, batch {B} (reduced config 5)",
            "value": round(B / (step_ms * 1e-3), 1), "unit": "tok/s", "ms_per_step": round(step_ms, 3),
            "e2e": {"value": round(B * n / dec_s, 1), "unit": "tok/s"},
            "prefill": {"tokens": 512 * B, "ms": round(prefill_ms, 2), "tok_s": round(512 * B / (prefill_ms * 1e-3), 1)},
            "model_file_s": round(gen_s, 1),
            "kernel_ms_per_step": {k: round(v[0], 3) for k, v in prof.items()},
            "roofline": {"bound": "hbm", "bytes_per_step": w_bytes + kv,
                         "achieved": round((w_bytes + kv) / (step_ms * 1e-3) / 1e9, 1), "peak": peak, "unit": "GB/s",
                         "frac": round((w_bytes + kv) / (step_ms * 1e-3) / 1e9 / peak, 4), "peak_source": peak_src}}


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


def run_quantize(args):
    """The GPU Q8_0 quantizer (scripts/quantize.py's quantize_q8) on the 7B shape's
    w1 + w3 of 4 layers as one flat tensor (4 x 2 x 11008 x 4096 = 360.7 M weights, 1.44 GB
    fp32 in, 406 MB out: larger than L2, so no flush between launches).
    value = weights/s of the device pass (CUDA events on the launching stream);
    e2e = nr_quantize_q8 from/to host numpy buffers (pinned-slot pipeline, H2D/D2H in the
    timed region); roofline: 5.125 algorithmic bytes per weight (4 read, 1.125 written)
    against the measured HBM copy bandwidth; cpu_baseline: the CPU restatement
    (oracle/nitro_oracle.cpp, one thread) on a bounded sample."""
    import torch
    from nitrorag_b200 import quantize_q8, quantized_size
    from nitrorag_b200._lib import lib
    peak, peak_src = load_peaks()
    n = 4 * 2 * 11008 * 4096
    g = torch.Generator(device="cuda").manual_seed(5)
    w = torch.randn(n, generator=g, device="cuda", dtype=torch.float32) * 0.02
    out = torch.empty(quantized_size(n), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()

    def launch():
        rc = lib().nr_quantize_q8_device(w.data_ptr(), n, out.data_ptr(), stream.cuda_stream)
        assert rc == 0, rc

    for _ in range(args.warmup):
        launch()
    torch.cuda.synchronize()
    e0, e1 = _dev_events(torch, stream)
    e0.record(stream)
    for _ in range(args.steps):
        launch()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    algo = 5.125 * n
    # e2e through host buffers: a 64 M-weight tensor (256 MB in), two runs
    n_h = 64 << 20
    w_h = w[:n_h].cpu().numpy()
    quantize_q8(w_h[: 1 << 20])
    t0 = time.perf_counter()
    reps = 2
    for _ in range(reps):
        host_out = quantize_q8(w_h)
    e2e_s = (time.perf_counter() - t0) / reps
    line = {"workload": "quantize", "metric": "Q8_0 quantize weights/s (scripts/quantize.py quantize_q8)",
            "value": round(n / (ms * 1e-3) / 1e9, 2), "unit": "Gweights/s", "ms_per_step": round(ms, 4),
            "higher_is_better": True, "dtype": "f32->q8_0", "data": "synthetic",
            "config": {"workload": "quantize", "weights": n, "flush": "inputs 1.44 GB > L2"},
            "e2e": {"value": round(n_h / e2e_s / 1e9, 3), "unit": "Gweights/s", "weights": n_h,
                    "h2d_bytes_per_step": 4 * n_h, "d2h_bytes_per_step": len(host_out)},
            "roofline": {"bound": "hbm", "achieved": round(algo / (ms * 1e-3) / 1e9, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(algo / (ms * 1e-3) / 1e9 / peak, 4),
                         "bytes_per_weight": 5.125, "peak_source": peak_src},
            "gpu_launches": args.steps, "steps": args.steps, "warmup": args.warmup}
    if not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle
        r = oracle.Restatement()
        n_c = 16 << 20
        sample = w_h[:n_c]
        t0 = time.perf_counter()
        r.quantize_q8(sample)
        cpu_s = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": round(n_c / cpu_s / 1e9, 4), "unit": "Gweights/s", "cores": 1,
                                "kind": "port", "sample": f"{n_c} weights through orc_quantize_q8 (scalar C)"}
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["engine", "reference"], default="engine")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-range", action="store_true",
                    help="mark the timed device-resident replays as the CUDA profiler range")
    ap.add_argument("--workload", choices=["decode64", "config1", "config3", "config4", "config5", "quantize"],
                    default="decode64", help="decode64 is the headline; the others print their own line")
    ap.add_argument("--batch", type=int, default=0, help="config5: requests per GPU (default 64)")
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
    if args.workload != "decode64":
        if rank == 0:
            fn = {"config1": run_config1, "config3": run_config3, "config4": run_config4,
                  "config5": run_config5, "quantize": run_quantize}[args.workload]
            print(json.dumps(fn(args)), flush=True)
        return 0
    return engine_arm(args, rank, world, local_rank)


if __name__ == "__main__":
    sys.exit(main())
