"""NR_SCHED_PACKED on a host-only engine: several prompt chunks per step within the token
budget, FIFO order, and admission by free pages (a request whose prompt does not fit
waits instead of exhausting the pool).  No reference counterpart: the reference admits one
chunk per step (src/pagedMemory.hpp:344-375), whose behaviour NR_SCHED_REFERENCE keeps
(tests/test_host_engine.py)."""
import pytest

from nitrorag_b200 import NR_SCHED_PACKED, NR_SCHED_REFERENCE, EngineConfig, NitroEngine, NrError

TINY_SHAPE = (128, 256, 2, 2, 2, 512, 512)


def host_engine(total_blocks, mode, max_new=20, budget=256):
    cfg = EngineConfig(total_blocks=total_blocks, max_new_tokens=max_new, max_tokens_per_batch=budget, device=-1,
                       sched_mode=mode)
    return NitroEngine(config=cfg, shape=TINY_SHAPE)


def _commit_all(eng, p, tok=1):
    n = sum(1 for part in p["prefills"] if part["done"]) + len(p["decode_req_ids"])
    eng.step_commit([tok] * n)


def test_several_chunks_per_step_within_budget():
    eng = host_engine(160, NR_SCHED_PACKED, max_new=4)
    for rid, n in enumerate([30, 40, 50, 300]):
        eng.add_request(rid, [rid + 3] * n)
    p = eng.step_plan()
    assert [(x["req_id"], x["start"], x["tokens"], x["done"]) for x in p["prefills"]] == [
        (0, 0, 30, True), (1, 0, 40, True), (2, 0, 50, True), (3, 0, 136, False)]
    assert p["prefill_req_id"] == 0 and p["prefill_tokens"] == 30 and p["decode_req_ids"] == []
    with pytest.raises(NrError):
        eng.step_commit([1, 2])  # three prompts completed: three tokens
    eng.step_commit([5, 6, 7])
    p = eng.step_plan()
    # decode rows take budget first; the last prompt's remaining 164 tokens fit in 253
    assert p["decode_req_ids"] == [0, 1, 2]
    assert [(x["req_id"], x["start"], x["tokens"], x["done"]) for x in p["prefills"]] == [(3, 136, 164, True)]
    _commit_all(eng, p)
    assert eng.request_tokens(3) == [1] and eng.request_tokens(0) == [5, 1]
    eng.close()


def test_reference_mode_admits_one_chunk():
    eng = host_engine(160, NR_SCHED_REFERENCE)
    for rid, n in enumerate([30, 40]):
        eng.add_request(rid, [9] * n)
    p = eng.step_plan()
    assert [(x["req_id"], x["tokens"]) for x in p["prefills"]] == [(0, 30)]
    eng.close()


def _run(eng, limit=200):
    steps = 0
    while eng.has_active_requests():
        _commit_all(eng, eng.step_plan())
        steps += 1
        assert steps < limit
    return steps


def test_admission_waits_for_pages():
    """12 pages; two 100-token prompts need 7 pages each.  Packed mode admits the second
    only after the first finished and released its pages; the reference's one-chunk-per-
    step admission runs out of pages instead."""
    eng = host_engine(12, NR_SCHED_PACKED, max_new=5)
    eng.add_request(0, list(range(100)))
    eng.add_request(1, list(range(200, 300)))
    p = eng.step_plan()
    assert [x["req_id"] for x in p["prefills"]] == [0]
    _commit_all(eng, p)
    for _ in range(4):  # request 0 decodes; request 1 still does not fit
        p = eng.step_plan()
        assert p["prefills"] == [] and p["decode_req_ids"] == [0]
        _commit_all(eng, p)
    _run(eng)
    assert len(eng.request_tokens(0)) == 5 and len(eng.request_tokens(1)) == 5

    ref = host_engine(12, NR_SCHED_REFERENCE, max_new=5)
    ref.add_request(0, list(range(100)))
    ref.add_request(1, list(range(200, 300)))
    with pytest.raises(NrError) as ei:
        _run(ref)
    assert ei.value.code == -5  # NR_ERR_NO_BLOCKS
    ref.close()
    eng.close()


def test_lone_request_is_admitted_even_if_it_cannot_fit():
    """With nothing running the head is admitted regardless of the estimate (otherwise it
    would wait forever); the allocation then reports the exhausted pool."""
    eng = host_engine(4, NR_SCHED_PACKED)
    eng.add_request(0, list(range(100)))
    with pytest.raises(NrError) as ei:
        eng.step_plan()
    assert ei.value.code == -5
    eng.close()


def test_many_small_requests_drain():
    eng = host_engine(64, NR_SCHED_PACKED, max_new=3, budget=64)
    for rid in range(40):
        eng.add_request(rid, [rid % 50 + 1] * (5 + rid % 13))
    steps = _run(eng)
    assert all(len(eng.request_tokens(r)) == 3 for r in range(40))
    assert steps < 40 * 3  # several admissions per step
    # every page is back: free, or cached and unreferenced
    assert len(eng.free_list()) + len(set(eng.cache_entries().values())) == 64
    eng.close()


def test_prefix_hits_for_several_admissions_in_one_step():
    """Two requests sharing a finished request's 48-token prefix are admitted in the same
    step; both map its three cached pages (the dry-run scan of the admission rule and the
    real scan agree), and neither sees the other's pages, allocated after admission."""
    eng = host_engine(64, NR_SCHED_PACKED, max_new=2)
    shared = list(range(100, 148))
    eng.add_request(0, shared + [7] * 20)
    _run(eng)  # request 0 finishes; its full pages stay in the prefix cache
    eng.add_request(1, shared + [8] * 10)
    eng.add_request(2, shared + [9] * 30)
    p = eng.step_plan()
    assert [(x["req_id"], x["start"], x["tokens"]) for x in p["prefills"]] == [(1, 48, 10), (2, 48, 30)]
    assert p["prefill_hits"] == 6
    t1, t2 = eng.request_block_table(1), eng.request_block_table(2)
    assert t1[:3] == t2[:3] and len(set(t1[3:]) & set(t2[3:])) == 0
    _commit_all(eng, p)
    eng.close()


def test_budget_split_between_decode_rows_and_chunks():
    """Decode rows take their budget first; the FIFO head then gets what is left and
    admission stops at a head it cannot finish."""
    eng = host_engine(256, NR_SCHED_PACKED, max_new=50, budget=64)
    for rid in range(3):
        eng.add_request(rid, [rid + 1] * 10)
    _commit_all(eng, eng.step_plan())  # three prompts of 10 in one step
    eng.add_request(3, [5] * 100)
    eng.add_request(4, [6] * 5)
    p = eng.step_plan()
    assert p["decode_req_ids"] == [0, 1, 2]
    assert [(x["req_id"], x["tokens"], x["done"]) for x in p["prefills"]] == [(3, 61, False)]
    _commit_all(eng, p)
    p = eng.step_plan()
    assert [(x["req_id"], x["start"], x["tokens"], x["done"]) for x in p["prefills"]] == [
        (3, 61, 39, True), (4, 0, 5, True)]
    eng.close()


@pytest.mark.parametrize("seed", range(6))
def test_packed_invariants_fuzz(seed):
    """Random workloads (prompt lengths, shared prefixes, budget, pool size, generation
    length): every step stays within the token budget, chunks are admitted in FIFO order
    and each request's chunks are contiguous, and a run either drains every request or
    stops with NR_ERR_NO_BLOCKS (decode growth can still exhaust a small pool)."""
    import random
    rnd = random.Random(seed)
    budget = rnd.choice([16, 64, 256])
    total = rnd.choice([24, 64, 400])
    max_new = rnd.choice([1, 3, 9])
    eng = host_engine(total, NR_SCHED_PACKED, max_new=max_new, budget=budget)
    shared = [rnd.randrange(512) for _ in range(32)]
    n_req = rnd.randint(5, 25)
    prompts = {}
    for rid in range(n_req):
        n = rnd.randint(1, 150)
        p = (shared + [rnd.randrange(512) for _ in range(n)]) if rnd.random() < 0.4 else [rnd.randrange(512) for _ in range(n)]
        prompts[rid] = p
        eng.add_request(rid, p)
    next_start = {rid: None for rid in prompts}
    admitted_order = []
    steps = 0
    try:
        while eng.has_active_requests():
            p = eng.step_plan()
            used = sum(x["tokens"] for x in p["prefills"]) + len(p["decode_req_ids"])
            assert used <= budget, (steps, used)
            for x in p["prefills"]:
                rid = x["req_id"]
                if rid not in admitted_order:
                    admitted_order.append(rid)
                if next_start[rid] is not None:
                    assert x["start"] == next_start[rid], (steps, rid)
                next_start[rid] = x["start"] + x["tokens"]
                assert x["done"] == (next_start[rid] == len(prompts[rid])), (steps, rid)
            _commit_all(eng, p, tok=rnd.randrange(512))
            steps += 1
            assert steps < 5000
    except NrError as err:
        assert err.code == -5, err
    else:
        assert all(len(eng.request_tokens(r)) == max_new for r in prompts if next_start[r] is not None)
    assert admitted_order == sorted(admitted_order)  # FIFO
    eng.close()


def test_admission_reserves_pages_to_finish():
    """Ten 60-token prompts generating 40 tokens each end at 99 tokens, 7 pages, so a
    40-page pool holds five at a time.  Their prompts alone (4 pages each) would all fit;
    packed admission reserves the pages each admitted request can still take, so at most
    five run at once and the run drains without NR_ERR_NO_BLOCKS."""
    eng = host_engine(40, NR_SCHED_PACKED, max_new=40, budget=1024)
    for rid in range(10):
        eng.add_request(rid, [rid + 1] * 60)
    most = 0
    steps = 0
    while eng.has_active_requests():
        _commit_all(eng, eng.step_plan())
        most = max(most, len(eng.running_batch()))
        steps += 1
        assert steps < 500
    assert most == 5
    assert all(len(eng.request_tokens(r)) == 40 for r in range(10))
    eng.close()


def test_reservation_capped_at_seq_len():
    """A generation length beyond the model's sequence length (512 here) reserves only up
    to seq_len: two 100-token prompts with max_new_tokens 100000 reserve 32 pages each,
    so a 64-page pool admits both in one step."""
    eng = host_engine(64, NR_SCHED_PACKED, max_new=100000, budget=1024)
    eng.add_request(0, [3] * 100)
    eng.add_request(1, [4] * 100)
    p = eng.step_plan()
    assert [x["req_id"] for x in p["prefills"]] == [0, 1]
    eng.close()
