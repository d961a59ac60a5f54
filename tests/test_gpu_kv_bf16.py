"""K/V pages in bf16 (NR_KV_BF16, off by default): every K/V value rounded to bf16 when it
is appended, attention still in fp32.  The reference keeps fp32 pages, so this option is
not parity with it.  Rounding to 8 significant bits is discontinuous: two correct fp32
computations that differ by ~1e-5 can store values one bf16 step (2^-8 relative) apart.
So the checks are:

* pages: every stored value exactly a bf16 number (the rounding happened); layer 0
  within one bf16 step of the CPU restatement run with the same rounding
  (orc_model_set_kv_bf16); deeper layers, which inherit earlier flips through attention,
  within 5 % of the pages' RMS;
* logits against that restatement within 1e-2 of the logits' RMS, and closer to it (in
  RMS) than to the fp32 reference (ref_fixed), i.e. the engine rounds where the
  restatement does;
* logits against the fp32 reference within 2e-2 of their RMS, the error bf16 pages bring;
* greedy tokens equal to the restatement's unless its two logits are within 1e-2 of the
  RMS of each other (then reported as a near tie under bf16 rounding)."""
import os

import numpy as np
import pytest

from nitrorag_b200 import NR_KV_BF16, NR_SCHED_PACKED, EngineConfig, NitroEngine, synth
from test_gpu_model import _check_tokens

pytestmark = pytest.mark.gpu


def _rms(x):
    return float(np.sqrt(np.mean(np.asarray(x, np.float64) ** 2)))


def _greedy(row):
    return int(np.argmax(np.where(row > 0, row, -np.inf))) if row.max() > 0 else 0


def _check_logits(le, want, lr, what):
    le, want, lr = (np.asarray(v, np.float64) for v in (le, want, lr))
    scale = _rms(want)
    assert np.max(np.abs(le - want)) <= 1e-2 * scale, f"{what}: vs bf16 restatement"
    assert np.max(np.abs(le - lr)) <= 2e-2 * _rms(lr), f"{what}: vs fp32 reference"
    d_bf16, d_fp32 = _rms(le - want), _rms(le - lr)
    assert d_bf16 <= d_fp32, f"{what}: closer to fp32 ({d_fp32:.3e}) than to the bf16 restatement ({d_bf16:.3e})"


def _check_token(got, row, what):
    want = _greedy(row)
    if got != want and abs(float(row[got]) - float(row[want])) > 1e-2 * _rms(row):
        _check_tokens(got, want, row, what)


def _check_pages(k_eng, k_orc, what):
    """Pages are [layer][16][kv_dim].  Every value must be a bf16 number.  Layer 0's values
    come from the same inputs on both sides (up to ~1e-5 of projection noise), so they must
    be within one bf16 step (plus 1e-3 of the RMS for values near zero); deeper layers
    inherit the flips of earlier ones through attention and are bounded in RMS."""
    bits = np.ascontiguousarray(k_eng, np.float32).view(np.uint32).ravel()
    assert np.all((bits & 0xFFFF) == 0), f"{what}: a stored value is not a bf16 number"
    a, b = np.asarray(k_eng, np.float64), np.asarray(k_orc, np.float64)
    a0, b0 = a[0].ravel(), b[0].ravel()
    step = 2.0 ** -7 * np.maximum(np.abs(a0), np.abs(b0)) + 1e-3 * float(np.sqrt(np.mean(b0 ** 2)))
    assert np.all(np.abs(a0 - b0) <= step), f"{what}: a layer-0 value more than one bf16 step away"
    assert _rms(a - b) <= 0.05 * _rms(b), f"{what}: pages differ by {_rms(a - b) / _rms(b):.3f} of their RMS"


def _run(path, restatement, ref, lens, decode_steps, seed, pages=256):
    eng = NitroEngine(path, EngineConfig(total_blocks=pages, max_new_tokens=64, max_batch=128, max_prefill_tokens=512,
                                         kv_dtype=NR_KV_BF16))
    model = restatement.model(path, pages)
    model.set_kv_bf16(True)
    ref.open(path, 512, pages)
    rng = np.random.default_rng(seed)
    V = eng.vocab_size
    seqs, rh, toks, pos = [], [], [], []
    for i, n in enumerate(lens):
        prompt = rng.integers(0, V, n).astype(np.int32)
        s = eng.seq_create(i)
        seqs.append(s)
        rh.append(ref.new_request(i, prompt))
        le, tok = eng.forward_prefill_chunk(s, prompt, 0)
        want = model.forward_prefill(eng.block_table(s), prompt, 0)
        lr = ref.forward_prefill(rh[i], prompt, 0)
        _check_logits(le, want, lr, f"bf16-page prefill seq {i} ({n} tokens)")
        toks.append(tok)
        pos.append(n)
    for step in range(decode_steps):
        # the engine allocates each row's token first; the restatement then uses its tables
        le, am = eng.forward_decode_batch(toks, pos, seqs)
        want = model.forward_decode([eng.block_table(s) for s in seqs], toks, pos)
        lr = ref.forward_decode(toks, pos, rh)
        for i in range(len(seqs)):
            _check_logits(le[i], want[i], lr[i], f"bf16-page decode step {step} row {i}")
            _check_token(int(am[i]), want[i], f"bf16-page decode step {step} row {i}")
        # the restatement and the reference continue with the engine's tokens
        toks = [int(t) for t in am]
        pos = [p + 1 for p in pos]
    for blk in eng.block_table(seqs[0])[:3]:
        k1, v1 = model.page(blk)
        k2, v2 = eng.read_page(blk)
        _check_pages(k2, k1, f"K page {blk}")
        _check_pages(v2, v1, f"V page {blk}")
    eng.close()
    model.close()
    ref.close()


@pytest.mark.parametrize("shape_args", [None, (256, 512, 2, 2, 1, 512, 1024)], ids=["tiny-hd64", "hd128-gqa2"])
def test_bf16_pages_many_rows(restatement, ref_fixed, tiny_model, model_dir, shape_args):
    """80 prompts of 1-60 tokens (prefill on the matvec and the tensor-core projections, K/V
    appended by both), then decode at B = 80: more (sequence, head) pairs than SMs, so the
    split decode kernel and its merge read the bf16 pages."""
    if shape_args is None:
        path = tiny_model
    else:
        path = synth.write_model(os.path.join(model_dir, "bf16_hd128.bin"), synth.ModelShape(*shape_args), seed=6)
    lens = [int(n) for n in np.random.default_rng(3).integers(1, 61, 80)]
    _run(path, restatement, ref_fixed, lens, 3, seed=70, pages=512)


@pytest.mark.parametrize("shape_args", [None, (256, 512, 2, 2, 1, 512, 1024)], ids=["tiny-hd64", "hd128-gqa2"])
def test_bf16_pages_small_batch(restatement, ref_fixed, tiny_model, model_dir, shape_args):
    """A 300-token prompt and two short ones, then decode at B = 3 (one attention CTA per
    (sequence, head) reading bf16 pages)."""
    if shape_args is None:
        path = tiny_model
    else:
        path = synth.write_model(os.path.join(model_dir, "bf16_hd128.bin"), synth.ModelShape(*shape_args), seed=6)
    _run(path, restatement, ref_fixed, [300, 17, 64], 8, seed=71)


def test_bf16_pages_110m(restatement, ref_fixed, m110_model):
    """The 110M model: a 24-token prompt on the tensor-core path, then decode at B = 1."""
    _run(m110_model, restatement, ref_fixed, [24], 3, seed=72, pages=64)


@pytest.mark.parametrize("B", [4, 24])
def test_bf16_pages_large_matrix_paths(restatement, ref_fixed, m110_model, monkeypatch, B):
    """The 110M model with every projection on the large-matrix paths (tile threshold at
    zero): prompts of 16-60 tokens prefilled through the stream-K kernel, then decode at
    B = 4 (int8 digit-plane kernel) or B = 24 (stream-K), K/V appended in bf16 by those
    kernels' epilogue."""
    monkeypatch.setenv("NITRO_TILE_MAX_WEIGHTS", "0")
    lens = [int(n) for n in np.random.default_rng(B).integers(16, 61, B)]
    _run(m110_model, restatement, ref_fixed, lens, 2, seed=73 + B, pages=512)


def test_bf16_pages_packed_scheduler(restatement, tiny_model):
    """NR_SCHED_PACKED with bf16 pages: several prompts in one forward pass (the tensor-core
    prefill attention over a segment table reads bf16 pages), each request's logits
    against the restatement with bf16 rounding."""
    eng = NitroEngine(tiny_model, EngineConfig(total_blocks=256, max_new_tokens=2, max_batch=32,
                                               max_tokens_per_batch=1024, max_prefill_tokens=1024,
                                               sched_mode=NR_SCHED_PACKED, kv_dtype=NR_KV_BF16))
    model = restatement.model(tiny_model, 256)
    model.set_kv_bf16(True)
    rng = np.random.default_rng(73)
    prompts = [rng.integers(0, 512, n).astype(np.int32) for n in (300, 200, 150, 40)]
    for i, p in enumerate(prompts):
        eng.add_request(i, p)
    res = eng.step(want_logits=True)
    assert res.n_prefill == 4
    for k, (rid, _) in enumerate(res.emitted):
        want = model.forward_prefill(eng.request_block_table(rid), prompts[rid], 0)
        assert np.max(np.abs(res.logits[k] - want)) <= 1e-2 * _rms(want), f"packed bf16-page prefill req {rid}"
    eng.close()
    model.close()
