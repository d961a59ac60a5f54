"""Model-level parity on the GPU: the engine (through its C ABI) against the reference's own
code compiled from its sources (oracle/_ref), on identical seeded model files.

Bit-exact: block tables, free lists, prefix-cache hits, greedy token ids.
Within RTOL/ATOL (1e-3 relative, 1e-4 absolute): logits.
`fixed` engine mode is checked against the ref_fixed build, `faithful` mode against the
unmodified reference (whose batched Q8 matmul keeps only the last 32-wide block)."""
import os

import numpy as np
import pytest

from conftest import assert_close
from nitrorag_b200 import NR_Q8_FAITHFUL, NR_Q8_FIXED, NR_SCHED_PACKED, EngineConfig, NitroEngine, synth

pytestmark = pytest.mark.gpu


def _engine(path, q8_mode=NR_Q8_FIXED, total_blocks=64, max_new=20, max_batch=64, max_prefill=256):
    return NitroEngine(path, EngineConfig(total_blocks=total_blocks, max_new_tokens=max_new, q8_mode=q8_mode,
                                          max_batch=max_batch, max_prefill_tokens=max_prefill))


def _margin(lg):
    s = np.sort(lg)
    return float(s[-1] - s[-2])


def _check_tokens(got, want, logits, what):
    """Token ids must match; a mismatch inside the logit tolerance is reported as a near tie."""
    if got != want:
        m = _margin(logits)
        raise AssertionError(f"{what}: token {got} != reference {want} (top-2 margin {m:.3e}"
                             f"{', a near tie' if m < 1e-3 else ''})")


@pytest.mark.parametrize("mode", ["fixed", "faithful"])
def test_sequence_api_prefill_decode(request, tiny_model, mode):
    ref = request.getfixturevalue("ref_fixed" if mode == "fixed" else "ref_faithful")
    ref.open(tiny_model, 256, 96)
    eng = _engine(tiny_model, NR_Q8_FIXED if mode == "fixed" else NR_Q8_FAITHFUL, total_blocks=96)
    rng = np.random.default_rng(3)
    lens = [40, 16, 77]
    rh, eh, toks, pos = [], [], [], []
    for i, n in enumerate(lens):
        prompt = rng.integers(0, ref.vocab, n).astype(np.int32)
        rh.append(ref.new_request(i, prompt))
        eh.append(eng.seq_create(i))
        lr = ref.forward_prefill(rh[i], prompt, 0)
        le, am = eng.forward_prefill_chunk(eh[i], prompt, 0)
        assert eng.block_table(eh[i]) == ref.block_table(rh[i])
        assert_close(le, lr, what=f"prefill logits seq {i}")
        _check_tokens(am, ref.argmax(lr), lr, f"prefill token seq {i}")
        toks.append(am)
        pos.append(n)
    for step in range(12):
        lr = ref.forward_decode(toks, pos, rh)
        le, am = eng.forward_decode_batch(toks, pos, eh)
        for i in range(len(lens)):
            assert eng.block_table(eh[i]) == ref.block_table(rh[i]), (step, i)
            assert_close(le[i], lr[i], what=f"decode step {step} row {i}")
            _check_tokens(int(am[i]), ref.argmax(lr[i]), lr[i], f"decode step {step} row {i}")
        toks = [int(t) for t in am]
        pos = [p + 1 for p in pos]
    assert eng.free_list() == ref.free_list()
    # K/V pages hold the same values (layout converted back to the reference's)
    for blk in ref.block_table(rh[2]):
        k1, v1 = ref.kv_page(blk)
        k2, v2 = eng.read_page(blk)
        assert_close(k2, k1, what=f"K page {blk}")
        assert_close(v2, v1, what=f"V page {blk}")
    eng.close()
    ref.close()


def _run_scheduler_pair(ref, eng, prompts, max_new, check_logits=True):
    handles = {}
    for i, p in enumerate(prompts):
        handles[i] = ref.new_request(i, p)
        ref.sched_add(handles[i])
        eng.add_request(i, p)
    steps = 0
    while ref.sched_has_active():
        assert eng.has_active_requests()
        B = ref.sched_step(max_new)
        res = eng.step(want_logits=check_logits)
        assert res.n_decode == B, steps
        assert eng.running_batch() == ref.sched_running(), steps
        # decode rows: the last len(res.emitted)-B entries, in running-batch order
        dec = res.emitted[len(res.emitted) - B:] if B else []
        if B and check_logits:
            lr = ref.sched_decode_logits(B)
            le = res.logits[len(res.emitted) - B:]
            for r in range(B):
                assert_close(le[r], lr[r], what=f"step {steps} decode row {r}")
        for r, (rid, tok) in enumerate(dec):
            want = ref.generated(handles[rid])[-1]
            if tok != want and check_logits:
                _check_tokens(tok, want, ref.sched_decode_logits(B)[r], f"step {steps} req {rid}")
            assert tok == want, (steps, rid)
        for rid, h in handles.items():
            assert eng.request_tokens(rid) == ref.generated(h), (steps, rid)
            assert eng.request_block_table(rid) == ref.block_table(h), (steps, rid)
        assert eng.free_list() == ref.free_list(), steps
        steps += 1
        assert steps < 10000
    assert not eng.has_active_requests()
    return steps


@pytest.mark.parametrize("mode", ["fixed", "faithful"])
def test_scheduler_with_prefix_sharing(request, tiny_model, mode):
    """Continuous_Scheduler::step end to end: 7 requests, 4 of them sharing a 48-token prefix
    (prefix-cache hits), one prompt longer than the 256-token budget (chunked prefill)."""
    ref = request.getfixturevalue("ref_fixed" if mode == "fixed" else "ref_faithful")
    ref.open(tiny_model, 256, 160)
    eng = _engine(tiny_model, NR_Q8_FIXED if mode == "fixed" else NR_Q8_FAITHFUL, total_blocks=160, max_new=9)
    rng = np.random.default_rng(17)
    V = ref.vocab
    shared = rng.integers(0, V, 48)
    prompts = []
    for i in range(7):
        if i in (1, 2, 4, 5):
            tail = rng.integers(0, V, int(rng.integers(1, 30)))
            prompts.append(np.concatenate([shared, tail]).astype(np.int32))
        elif i == 3:
            prompts.append(rng.integers(0, V, 300).astype(np.int32))
        else:
            prompts.append(rng.integers(0, V, int(rng.integers(5, 60))).astype(np.int32))
    _run_scheduler_pair(ref, eng, prompts, max_new=9)
    st = eng.stats()
    assert st["cache_hit_pages"] > 0
    eng.close()
    ref.close()


def test_scheduler_pool_pressure_eviction(ref_fixed, tiny_model):
    """A pool small enough that finished requests' cached pages are evicted (5% / 20% rule)."""
    ref = ref_fixed
    ref.open(tiny_model, 256, 32)
    eng = _engine(tiny_model, NR_Q8_FIXED, total_blocks=32, max_new=6)
    rng = np.random.default_rng(23)
    V = ref.vocab
    shared = rng.integers(0, V, 32)
    prompts = [np.concatenate([shared, rng.integers(0, V, 40)]).astype(np.int32) for _ in range(24)]
    _run_scheduler_pair(ref, eng, prompts, max_new=6)
    assert eng.stats()["evictions"] > 0
    eng.close()
    ref.close()


def test_110m_config1_prefill_and_decode(ref_fixed, m110_model):
    """BASELINE config 1 shape on the 110M model: 256-token prompt, then greedy decode
    (24 steps here; the bench runs the full 128)."""
    ref = ref_fixed
    ref.open(m110_model, 256, 64)
    eng = _engine(m110_model, NR_Q8_FIXED, total_blocks=64)
    rng = np.random.default_rng(1)
    prompt = rng.integers(0, 32000, 256).astype(np.int32)
    rh = ref.new_request(0, prompt)
    eh = eng.seq_create(0)
    lr = ref.forward_prefill(rh, prompt, 0)
    le, tok = eng.forward_prefill_chunk(eh, prompt, 0)
    assert_close(le, lr, what="110M prefill logits")
    _check_tokens(tok, ref.argmax(lr), lr, "110M prefill token")
    pos = 256
    for step in range(24):
        lr = ref.forward_decode([tok], [pos], [rh])
        le, am = eng.forward_decode_batch([tok], [pos], [eh])
        assert_close(le[0], lr[0], what=f"110M decode step {step}")
        _check_tokens(int(am[0]), ref.argmax(lr[0]), lr[0], f"110M decode step {step}")
        tok = int(am[0])
        pos += 1
    assert eng.block_table(eh) == ref.block_table(rh)
    eng.close()
    ref.close()


def test_110m_decode_batch_64(ref_fixed, m110_model):
    """The benchmark's decode batch: 64 sequences with ragged contexts, three steps."""
    ref = ref_fixed
    ref.open(m110_model, 256, 700)
    eng = _engine(m110_model, NR_Q8_FIXED, total_blocks=700)
    prompts = synth.decode_workload(64, 20, 150, 32000, seed=9)
    rh, eh, toks, pos = [], [], [], []
    for i, p in enumerate(prompts):
        rh.append(ref.new_request(i, p))
        eh.append(eng.seq_create(i))
        # prefill on the engine only; the reference reads the same K/V after a copy below
        lr = ref.forward_prefill(rh[i], p, 0)
        le, am = eng.forward_prefill_chunk(eh[i], p, 0)
        assert_close(le, lr, what=f"prefill {i}")
        toks.append(am)
        pos.append(len(p))
    for step in range(3):
        lr = ref.forward_decode(toks, pos, rh)
        le, am = eng.forward_decode_batch(toks, pos, eh)
        assert_close(le, lr, what=f"B=64 decode step {step}")
        for i in range(64):
            _check_tokens(int(am[i]), ref.argmax(lr[i]), lr[i], f"B=64 step {step} row {i}")
        toks = [int(t) for t in am]
        pos = [p + 1 for p in pos]
    eng.close()
    ref.close()


def test_forward_paged_matches_unmodified_reference(ref_faithful, tiny_model):
    """forward_paged (src/model_q8.cpp:244) uses the reference's correct single-token matmul
    even in the unmodified build: the engine's forward_paged must match it in any mode."""
    ref = ref_faithful
    ref.open(tiny_model, 256, 64)
    eng = _engine(tiny_model, NR_Q8_FAITHFUL, total_blocks=64)
    rng = np.random.default_rng(4)
    prompt = rng.integers(0, ref.vocab, 33).astype(np.int32)
    rh = ref.new_request(0, prompt)
    eh = eng.seq_create(0)
    ref.forward_prefill(rh, prompt, 0)
    eng.forward_prefill_chunk(eh, prompt, 0)
    tok, pos = 100, 33
    for step in range(6):
        lr = ref.forward_paged(rh, tok, pos)
        le, am = eng.forward_paged(eh, tok, pos)
        assert_close(le, lr, what=f"forward_paged step {step}")
        pos += 1
    eng.close()
    ref.close()


def test_ingest_prompt_prefix_cache_hit(ref_fixed, tiny_model):
    """Bench Exp 4 (src/model_q8.cpp:910-939): the same prompt twice with flush_cache; the
    second ingest maps every page from the cache and computes nothing."""
    ref = ref_fixed
    ref.open(tiny_model, 256, 64)
    eng = _engine(tiny_model, NR_Q8_FIXED, total_blocks=64)
    prompt = np.full(64, 263 % ref.vocab, np.int32)
    ra, rb = ref.new_request(1, []), ref.new_request(2, [])
    ea, eb = eng.seq_create(1), eng.seq_create(2)
    n_r, lg_r = ref.ingest_prompt(ra, prompt, True)
    n_e, comp, lg_e = eng.ingest_prompt(ea, prompt, True)
    assert n_r == n_e == 64 and comp == 64
    assert_close(lg_e, lg_r, what="ingest miss logits")
    ref.flush(ra)
    eng.flush_cache(ea)
    n_r, _ = ref.ingest_prompt(rb, prompt, True)
    n_e, comp, _ = eng.ingest_prompt(eb, prompt, True)
    assert n_r == n_e == 64 and comp == 0
    assert eng.block_table(eb) == ref.block_table(rb) == ref.block_table(ra)
    assert eng.free_list() == ref.free_list()
    for i in range(64):
        assert eng.block_state(i) == ref.block_state(i)
    eng.close()
    ref.close()


@pytest.mark.parametrize("wide", [True, False], ids=["hilo-tiles", "raw-tiles"])
@pytest.mark.parametrize("B", [1, 3, 5, 8, 10, 24, 40, 64])
def test_110m_raw_q8_tiles(ref_fixed, m110_model, monkeypatch, B, wide):
    """The large-model projection path: with the tile threshold at zero every Q8 projection
    gets raw Q8 tiles, and hi/lo tiles beside them unless NITRO_WIDE_TILES=0.  Batches of
    1-10 rows take the int8 digit-plane kernel (the raw tiles straight into kind::i8
    MMAs, 16 or 32 columns), 11-64 rows the stream-K kernel (over the hi/lo tiles when
    they exist, else converting the raw ones); both cut these small matrices' tiles over
    up to 12 CTAs each, so the partial-tile hand-over runs on every projection.  Prefill and two decode steps must match the
    reference, and a decode step run again on the same inputs must give bit-identical
    logits (partials are added in a fixed order)."""
    monkeypatch.setenv("NITRO_TILE_MAX_WEIGHTS", "0")
    monkeypatch.setenv("NITRO_WIDE_TILES", "1" if wide else "0")
    ref = ref_fixed
    blocks = 600
    ref.open(m110_model, 256, blocks)
    eng = _engine(m110_model, NR_Q8_FIXED, total_blocks=blocks)
    prompts = synth.decode_workload(B, 20, 90, 32000, seed=12 + B)
    rh, eh, toks, pos = [], [], [], []
    for i, p in enumerate(prompts):
        rh.append(ref.new_request(i, p))
        eh.append(eng.seq_create(i))
        lr = ref.forward_prefill(rh[i], p, 0)
        le, am = eng.forward_prefill_chunk(eh[i], p, 0)
        assert_close(le, lr, what=f"raw-tile prefill {i}")
        toks.append(am)
        pos.append(len(p))
    for step in range(2):
        lr = ref.forward_decode(toks, pos, rh)
        le, am = eng.forward_decode_batch(toks, pos, eh)
        assert_close(le, lr, what=f"raw-tile B={B} decode step {step}")
        if step == 0:  # the same step again: same K/V rows rewritten, same logits bit for bit
            le2, am2 = eng.forward_decode_batch(toks, pos, eh)
            assert np.array_equal(le2, le) and np.array_equal(am2, am)
        for i in range(B):
            _check_tokens(int(am[i]), ref.argmax(lr[i]), lr[i], f"raw-tile B={B} step {step} row {i}")
        toks = [int(t) for t in am]
        pos = [p + 1 for p in pos]
    eng.close()
    ref.close()


def test_head_dim_128_prefill_decode(ref_fixed, model_dir):
    """head_dim 128 (the 7B shape's heads) on a small model: prefill chunks of 1-130 tokens
    through the causal attention (4 queries per warp at this head size), then decode,
    against the reference."""
    shape = synth.ModelShape(256, 512, 2, 2, 2, 512, 512)
    path = synth.write_model(os.path.join(model_dir, "hd128.bin"), shape, seed=21)
    ref = ref_fixed
    ref.open(path, 256, 96)
    eng = _engine(path, NR_Q8_FIXED, total_blocks=96)
    rng = np.random.default_rng(8)
    lens = [1, 33, 130]
    rh, eh, toks, pos = [], [], [], []
    for i, n in enumerate(lens):
        prompt = rng.integers(0, ref.vocab, n).astype(np.int32)
        rh.append(ref.new_request(i, prompt))
        eh.append(eng.seq_create(i))
        lr = ref.forward_prefill(rh[i], prompt, 0)
        le, am = eng.forward_prefill_chunk(eh[i], prompt, 0)
        assert_close(le, lr, what=f"hd128 prefill logits seq {i}")
        toks.append(am)
        pos.append(n)
    for step in range(3):
        lr = ref.forward_decode(toks, pos, rh)
        le, am = eng.forward_decode_batch(toks, pos, eh)
        assert_close(le, lr, what=f"hd128 decode step {step}")
        toks = [int(t) for t in am]
        pos = [p + 1 for p in pos]
    eng.close()
    ref.close()


@pytest.mark.parametrize("shape_args", [(512, 1024, 2, 8, 2, 512, 1024), (256, 512, 2, 2, 1, 512, 1024)],
                         ids=["hd64-gqa4", "hd128-gqa2"])
def test_single_sequence_decode_grouped_kv(ref_fixed, model_dir, shape_args):
    """Batch-1 decode (one attention CTA per head, matvec projections) with grouped KV heads
    at both head sizes: a context that grows from 300 to 323 tokens (up to 21 pages, so the
    attention warps cycle their page rings), 24 greedy steps with logits against the
    reference."""
    shape = synth.ModelShape(*shape_args)
    path = synth.write_model(os.path.join(model_dir, f"b1_{shape.dim}_{shape.n_heads}.bin"), shape, seed=5)
    ref = ref_fixed
    ref.open(path, 512, 96)
    eng = _engine(path, NR_Q8_FIXED, total_blocks=96, max_new=32, max_batch=4, max_prefill=512)
    prompt = np.random.default_rng(12).integers(0, ref.vocab, 300).astype(np.int32)
    rh = ref.new_request(0, prompt)
    eh = eng.seq_create(0)
    lr = ref.forward_prefill(rh, prompt, 0)
    le, tok = eng.forward_prefill_chunk(eh, prompt, 0)
    assert_close(le, lr, what="prefill logits")
    pos = len(prompt)
    for step in range(24):
        lr = ref.forward_decode([tok], [pos], [rh])
        le, am = eng.forward_decode_batch([tok], [pos], [eh])
        assert_close(le[0], lr[0], what=f"decode step {step}")
        _check_tokens(int(am[0]), ref.argmax(lr[0]), lr[0], f"decode step {step}")
        tok = int(am[0])
        pos += 1
    assert eng.block_table(eh) == ref.block_table(rh)
    eng.close()
    ref.close()


def _packed_vs_reference(ref, eng, prompts, max_new, what):
    """Run the engine's NR_SCHED_PACKED steps to completion; every emitted logits row and
    token is checked against the reference computing that request alone (its prompt in
    one prefill, then one decode per token)."""
    rh = {}
    for i, p in enumerate(prompts):
        eng.add_request(i, p)
        rh[i] = ref.new_request(i, p)
    n_tok = {i: 0 for i in range(len(prompts))}
    steps = multi = 0
    while eng.has_active_requests():
        res = eng.step(want_logits=True)
        multi = max(multi, res.n_prefill)
        for k, (rid, tok) in enumerate(res.emitted):
            p = prompts[rid]
            if n_tok[rid] == 0:
                lr = ref.forward_prefill(rh[rid], p, 0)
            else:
                prev = eng.request_tokens(rid)[n_tok[rid] - 1]
                lr = ref.forward_decode([prev], [len(p) + n_tok[rid] - 1], [rh[rid]])[0]
            assert_close(res.logits[k], lr, what=f"{what}: step {steps} req {rid} token {n_tok[rid]}")
            _check_tokens(tok, ref.argmax(lr), lr, f"{what}: step {steps} req {rid} token {n_tok[rid]}")
            n_tok[rid] += 1
        steps += 1
        assert steps < 1000
    assert all(n == max_new for n in n_tok.values()), n_tok
    return multi


@pytest.mark.parametrize("shape_args", [None, (256, 512, 2, 2, 1, 512, 1024)], ids=["tiny-hd64", "hd128-gqa2"])
def test_packed_scheduler_multi_prompt_prefill(ref_fixed, tiny_model, model_dir, shape_args):
    """NR_SCHED_PACKED: several prompt chunks per step in one forward pass (rows
    concatenated through the projections, causal attention per chunk from a tile table),
    a prompt longer than the budget split across steps, against the reference run one
    request at a time."""
    if shape_args is None:
        path = tiny_model
    else:
        path = synth.write_model(os.path.join(model_dir, "packed_hd128.bin"), synth.ModelShape(*shape_args), seed=4)
    ref = ref_fixed
    ref.open(path, 512, 256)
    eng = NitroEngine(path, EngineConfig(total_blocks=256, max_new_tokens=6, max_batch=64, max_prefill_tokens=256,
                                         sched_mode=NR_SCHED_PACKED))
    rng = np.random.default_rng(31)
    lens = [5, 17, 33, 60, 300, 1, 48, 90, 130, 16]
    prompts = [rng.integers(0, ref.vocab, n).astype(np.int32) for n in lens]
    multi = _packed_vs_reference(ref, eng, prompts, 6, "packed")
    assert multi >= 3  # several chunks shared a forward pass
    eng.close()
    ref.close()


def test_packed_scheduler_110m(ref_fixed, m110_model):
    """The 110M model: chunks of up to 256 concatenated rows on the tensor-core projections."""
    ref = ref_fixed
    ref.open(m110_model, 512, 256)
    eng = NitroEngine(m110_model, EngineConfig(total_blocks=256, max_new_tokens=4, max_batch=64,
                                               max_prefill_tokens=256, sched_mode=NR_SCHED_PACKED))
    rng = np.random.default_rng(32)
    prompts = [rng.integers(0, 32000, n).astype(np.int32) for n in (40, 100, 70, 200, 23, 64)]
    multi = _packed_vs_reference(ref, eng, prompts, 4, "packed 110M")
    assert multi >= 2
    eng.close()
    ref.close()


def test_110m_long_prompt_in_chunks(ref_fixed, m110_model):
    """Causal prefill attention over chunks that start mid-page and mid query tile: a
    700-token prompt as chunks of 1, 299 and 400 tokens (positions 0, 1 and 300), the last
    logits of each chunk against the reference's prefill of the same chunks."""
    ref = ref_fixed
    ref.open(m110_model, 512, 64)
    eng = _engine(m110_model, NR_Q8_FIXED, total_blocks=64, max_prefill=512)
    prompt = np.random.default_rng(5).integers(0, 32000, 700).astype(np.int32)
    rh = ref.new_request(0, prompt)
    eh = eng.seq_create(0)
    start = 0
    for n in (1, 299, 400):
        chunk = prompt[start:start + n]
        lr = ref.forward_prefill(rh, chunk, start)
        le, tok = eng.forward_prefill_chunk(eh, chunk, start)
        assert_close(le, lr, what=f"chunk at {start}")
        _check_tokens(tok, ref.argmax(lr), lr, f"chunk at {start}")
        start += n
    assert eng.block_table(eh) == ref.block_table(rh)
    eng.close()
    ref.close()
