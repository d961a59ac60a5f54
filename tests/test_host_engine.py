"""Host logic of the engine without a GPU (host-only engine, nr_engine_create_host_only):
the paged KV allocator, prefix cache and reference-mode scheduler against the reference's
own classes (src/pagedMemory.hpp), bit for bit, plus the error paths that replace the
reference's exit(1)."""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN
from nitrorag_b200 import EngineConfig, NitroEngine, NrError, synth

TINY_SHAPE = (128, 256, 2, 2, 2, 512, 512)


def host_engine(total_blocks, max_new=20, shape=TINY_SHAPE):
    return NitroEngine(config=EngineConfig(total_blocks=total_blocks, max_new_tokens=max_new, device=-1), shape=shape)


def _assert_same_pool(ref, eng, total, live_pairs, step):
    assert ref.free_list() == eng.free_list(), step
    assert ref.lru() == eng.lru(), step
    assert ref.cache_entries() == eng.cache_entries(), step
    for i in range(total):
        assert ref.block_state(i) == eng.block_state(i), (step, i)
        assert ref.is_cached(i) == eng.is_cached(i), (step, i)
    for rh, eh in live_pairs:
        assert ref.block_table(rh) == eng.block_table(eh), step
        a, b = ref.seq_info(rh), eng.seq_info(eh)
        assert a == b, (step, a, b)


@pytest.mark.parametrize("seed,total", [(1, 40), (2, 24), (3, 64), (4, 200)])
def test_allocator_fuzz_against_reference(ref_faithful, seed, total):
    """Random allocate / flush / release sequences with heavily shared prefixes (cache hits,
    duplicate inserts, eviction under the 5% / 20% rule) against KVBlock_Manager,
    PrefixCacheManager and Sequence compiled from the reference."""
    ref = ref_faithful
    ref.pool_only(total, 1, 16)
    eng = host_engine(total)
    rng = np.random.default_rng(seed)
    prompts = [rng.integers(0, 50, 80) for _ in range(3)]
    rh, eh, live = [], [], []
    for step in range(2500):
        op = rng.integers(0, 10)
        if op < 2 and len(live) < 8:
            sid = len(rh)
            rh.append(ref.new_request(sid, []))
            eh.append(eng.seq_create(sid))
            live.append(sid)
        elif op < 8 and live:
            s = live[rng.integers(len(live))]
            n = ref.seq_info(rh[s])["logical_token_count"]
            p = prompts[s % 3]
            tok = int(p[n % len(p)]) if rng.random() < 0.9 else int(rng.integers(0, 50))
            if ref.free_count() == 0 and not ref.lru():
                continue  # the reference would exit(1) here; covered by test_pool_exhaustion
            ref.alloc_token(rh[s], tok)
            eng.allocate_next_token(eh[s], tok)
        elif op < 9 and live:
            s = live[rng.integers(len(live))]
            ref.flush(rh[s])
            eng.flush_cache(eh[s])
        elif live:
            s = live.pop(int(rng.integers(len(live))))
            ref.release(rh[s])
            eng.release(eh[s])
        if step % 7 == 0 or step > 2400:
            _assert_same_pool(ref, eng, total, [(rh[s], eh[s]) for s in live], step)
    ref.close()
    eng.close()


def test_prefix_hits_share_pages_by_refcount():
    """ingest of a cached prompt maps the same physical pages and bumps their refcounts."""
    eng = host_engine(64)
    a, b = eng.seq_create(1), eng.seq_create(2)
    prompt = list(range(48))
    for t in prompt:
        eng.allocate_next_token(a, t)
    eng.flush_cache(a)
    pages = eng.block_table(a)
    assert len(pages) == 3 and all(eng.is_cached(p) for p in pages)
    # the prefix-cache scan of ingest_prompt runs on the host; a full hit computes nothing
    n, computed, lg = eng.ingest_prompt(b, prompt, True)
    assert (n, computed, lg) == (48, 0, None)
    assert eng.block_table(b) == pages
    for p in pages:
        assert eng.block_state(p)[1] == 2  # ref_count
    eng.release(a)
    eng.release(b)
    for p in pages:
        assert eng.block_state(p)[1] == 0 and eng.is_cached(p)
    assert set(eng.lru()) == {pages[-1]}  # only the leaf is evictable
    eng.close()


def test_scheduler_trace_matches_reference_golden():
    """Continuous_Scheduler::step decisions (decode batch, running order, admission with
    prefix-cache hits, chunked prefill, releases) and every block table and free list, per
    step, against a trace of the reference; sampled tokens are taken from the trace."""
    trace = json.load(open(os.path.join(GOLDEN, "golden.json")))["scheduler"]
    eng = host_engine(trace["total_blocks"], max_new=trace["max_new"])
    prompts = trace["prompts"]
    for i, p in enumerate(prompts):
        eng.add_request(i, p)
    for k, st in enumerate(trace["steps"]):
        plan = eng.step_plan()
        assert len(plan["decode_req_ids"]) == st["B"], k
        toks = [t for _, t in st["emitted"]]
        ids = [r for r, _ in st["emitted"]]
        want_ids = ([plan["prefill_req_id"]] if plan["prefill_done"] else []) + plan["decode_req_ids"]
        assert ids == want_ids, k
        eng.step_commit(toks)
        assert eng.running_batch() == st["running"], k
        assert eng.free_list() == st["free_list"], k
        for rid in range(len(prompts)):
            assert eng.request_block_table(rid) == st["block_tables"][rid], (k, rid)
            assert eng.request_tokens(rid) == st["generated"][rid], (k, rid)
    assert not eng.has_active_requests() or eng.step_plan()["n_released"] > 0
    assert {str(h): b for h, b in eng.cache_entries().items()} == trace["cache_entries"]
    eng.close()


def test_chunked_prefill_budget():
    """A 300-token prompt is admitted in two chunks (256 then 44, the 256-token budget,
    src/pagedMemory.hpp:307,361); decode rows consume budget first."""
    eng = host_engine(160, max_new=3)
    eng.add_request(0, list(range(10, 40)))
    eng.add_request(1, [7] * 300)
    p = eng.step_plan()
    assert p["prefill_req_id"] == 0 and p["prefill_tokens"] == 30 and p["prefill_done"]
    eng.step_commit([5])
    p = eng.step_plan()
    assert p["decode_req_ids"] == [0] and p["prefill_req_id"] == 1 and p["prefill_tokens"] == 255
    assert not p["prefill_done"]
    eng.step_commit([6])
    p = eng.step_plan()
    assert p["prefill_tokens"] == 45 and p["prefill_done"] and p["prefill_start"] == 255
    eng.close()


def test_pool_exhaustion_is_an_error_not_exit():
    """The reference exits (src/pagedMemory.hpp:117,212); the engine returns NR_ERR_NO_BLOCKS."""
    eng = host_engine(4)
    s = eng.seq_create(0)
    for t in range(64):
        eng.allocate_next_token(s, t)
    with pytest.raises(NrError) as ei:
        eng.allocate_next_token(s, 64)
    assert ei.value.code == -5
    eng.close()


def test_pool_exhaustion_in_scheduler_step():
    eng = host_engine(4, max_new=100)
    eng.add_request(0, list(range(60)))
    eng.step_plan()
    eng.step_commit([1])
    with pytest.raises(NrError) as ei:
        for _ in range(10):
            p = eng.step_plan()
            eng.step_commit([1] * (int(p["prefill_done"]) + len(p["decode_req_ids"])))
    assert ei.value.code == -5
    eng.close()


def test_invalid_arguments(tmp_path):
    with pytest.raises(NrError) as ei:
        NitroEngine(str(tmp_path / "missing.bin"), EngineConfig(device=0))
    assert ei.value.code == -2
    bad = tmp_path / "short.bin"
    bad.write_bytes(synth.SHAPE_TINY.header() + b"\0" * 100)
    with pytest.raises(NrError) as ei:
        NitroEngine(str(bad), EngineConfig(device=0))
    assert ei.value.code == -3
    with pytest.raises(NrError) as ei:
        NitroEngine(config=EngineConfig(total_blocks=0, device=-1), shape=TINY_SHAPE)
    assert ei.value.code == -1
    eng = host_engine(8)
    with pytest.raises(NrError):
        eng.add_request(0, [])
    with pytest.raises(NrError):
        eng.add_request(1, [512])  # token id >= vocab
    with pytest.raises(NrError) as ei:
        eng.forward_prefill_chunk(eng.seq_create(0), [1, 2], 0)
    assert ei.value.code == -6  # host-only engine has no device
    for replay in (lambda: eng.replay_decode(1), lambda: eng.replay_decode_attention(1, True)):
        with pytest.raises(NrError) as ei:
            replay()
        assert ei.value.code == -6
    from nitrorag_b200._lib import lib
    assert lib().nr_replay_decode_attention(None, 1, 0) == -1
    assert lib().nr_replay_decode_attention(eng._h, -1, 0) == -1
    eng.close()
