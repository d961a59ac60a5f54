"""Replicas: one request stream served by N independent engines, one per GPU.

The model does not shard, so the multi-GPU path is N full replicas (weights, page pool,
prefix cache each) with requests partitioned on the host: request i of the arrival-ordered
stream goes to replica i mod N.  The split is deterministic, so each replica's request
stream, and therefore its scheduler trace, can be replayed by the reference on its own.
Nothing crosses between replicas on the data path; a launcher only gathers counts and
timings at the end.

``run_stream`` drives one engine (GPU or host-only) through its part of the stream with
the virtual clock the benchmark and the parity tests use: scheduler iteration k admits
every request whose arrival time is <= k * step_s."""
from __future__ import annotations

from dataclasses import dataclass, field


def partition(n_requests: int, world: int, rank: int) -> list[int]:
    """Indices (in arrival order) of the requests replica `rank` of `world` serves."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    return list(range(rank, n_requests, world))


@dataclass
class StreamResult:
    steps: int = 0
    generated: int = 0
    prefill_hits: int = 0
    decode_rows: int = 0
    prefill_tokens: int = 0
    tokens: dict = field(default_factory=dict)  # req id -> generated token ids


def run_stream(engine, arrivals, prompts, ids, step_s: float = 0.010, host_tokens=None, on_step=None,
               on_admit=None, id_offset: int = 0, max_steps: int = 1_000_000) -> StreamResult:
    """Serve the requests `ids` (indices into arrivals/prompts, arrival order) on `engine`.

    A GPU engine steps with nr_step.  A host-only engine steps with nr_step_plan /
    nr_step_commit and needs `host_tokens(plan) -> list of token ids` (one per chunk that
    completes its prompt, then one per decode row).  `on_step(k, result)` is called after
    every iteration that ran (k counts them), `on_admit(i)` after request i is added.
    Request ids are the global stream indices plus `id_offset`."""
    res = StreamResult()
    ids = list(ids)
    nxt, k = 0, 0
    gpu = engine.config.device >= 0
    while True:
        while nxt < len(ids) and arrivals[ids[nxt]] <= k * step_s:
            i = ids[nxt]
            engine.add_request(i + id_offset, prompts[i])
            if on_admit:
                on_admit(i)
            nxt += 1
        k += 1
        if not engine.has_active_requests():
            if nxt >= len(ids):
                break
            continue
        if gpu:
            r = engine.step()
            res.generated += len(r.emitted)
            res.prefill_hits += r.prefill_hits
            res.decode_rows += r.n_decode
            res.prefill_tokens += r.prefill_tokens
        else:
            plan = engine.step_plan()
            toks = host_tokens(plan)
            engine.step_commit(toks)
            r = plan
            res.generated += len(toks)
            res.prefill_hits += plan["prefill_hits"]
            res.decode_rows += len(plan["decode_req_ids"])
            res.prefill_tokens += sum(c["tokens"] for c in plan["prefills"])
        if on_step:
            on_step(res.steps, r)
        res.steps += 1
        if res.steps >= max_steps:
            raise RuntimeError("stream did not finish within max_steps")
    for i in ids:
        res.tokens[i] = engine.request_tokens(i + id_offset)
    return res
