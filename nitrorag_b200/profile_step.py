"""One engine step inside a CUDA profiler range, for capturing individual kernels with a
profiler started as `--profile-from-start off`:

    ncu --profile-from-start off --set full --clock-control none -k regex:tc_gemm -c 1 \\
        -o out python -m nitrorag_b200.profile_step [--batch B] [--prefill T]

Default: one decode step of 64 sequences of the 110M Q8_0 model (contexts U[128, 200],
1024-page pool, so the device holds ~1.7 GB: small enough for multi-pass captures, with
weights and K/V still far larger than L2).  `--batch B` decodes B sequences instead;
`--prefill T` instead profiles the prefill of one T-token prompt (T <= 1024, model
header with seq_len 2048).  `--wide` profiles one decode step of B one-token sequences
of a 2-layer model of the 7B shape's width (dim 4096, ffn 11008, 32 heads: ~2.5 GB on
the device), whose projections take the large-matrix kernels (stream-K, int8 digit
planes, ring matvec by batch width).  `--matvec` profiles two nr_q8_matmul launches at
one row over 22016 x 4096 (after two unprofiled ones).  The step runs eagerly (no CUDA
graph) so each kernel is an ordinary launch.
"""
from __future__ import annotations

import argparse
import os
import sys


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--prefill", type=int, default=0)
    ap.add_argument("--wide", action="store_true")
    ap.add_argument("--matvec", action="store_true")
    args = ap.parse_args()
    os.environ.setdefault("NITRO_GRAPHS", "0")
    import numpy as np
    import torch

    from . import EngineConfig, NitroEngine, synth

    rng = np.random.default_rng(3)
    if args.matvec:
        import ctypes as C

        from ._lib import NR_Q8_FIXED, lib
        N, K = 22016, 4096
        st = torch.cuda.current_stream()
        mats = [(torch.randint(-127, 128, (N, K), dtype=torch.int8, device="cuda"),
                 torch.rand((N, K // 32), device="cuda") * 1e-3) for _ in range(2)]
        x = torch.randn((1, K), device="cuda")
        out = torch.empty((1, N), device="cuda")
        for i in range(4):
            if i == 2:
                torch.cuda.synchronize()
                torch.cuda.profiler.start()
            q, s = mats[i % 2]
            assert lib().nr_q8_matmul(x.data_ptr(), q.data_ptr(), s.data_ptr(), out.data_ptr(), 1, N, K, NR_Q8_FIXED,
                                      C.c_void_p(st.cuda_stream)) == 0
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        print("profiled two 1 x 22016 x 4096 nr_q8_matmul launches")
        return 0
    if args.wide:
        B = max(1, min(args.batch, 64))
        shape = synth.ModelShape(4096, 11008, 2, 32, 32, 32000, 512)
        model = synth.cached_model_on_device(shape, seed=7)
        eng = NitroEngine(model, EngineConfig(total_blocks=B * 4 + 8, max_new_tokens=1000, max_batch=B,
                                              max_prefill_tokens=64, device=0))
        seqs = [eng.seq_create(i) for i in range(B)]
        toks = [int(eng.forward_prefill_chunk(s, [i + 1], 0, want_logits=False)[1]) for i, s in enumerate(seqs)]
        pos = [1] * B
        for _ in range(2):
            _, am = eng.forward_decode_batch(toks, pos, seqs, want_logits=False)
            toks, pos = [int(t) for t in am], [p + 1 for p in pos]
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        eng.forward_decode_batch(toks, pos, seqs, want_logits=False)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        print(f"profiled one decode step of {B} sequences of the 2-layer 7B-width model")
        return 0
    if args.prefill:
        T = min(args.prefill, 1024)
        model = synth.cached_model(synth.SHAPE_110M_LONG, seed=1234)
        eng = NitroEngine(model, EngineConfig(total_blocks=256, max_new_tokens=100000, max_batch=8,
                                              max_prefill_tokens=1024, device=0))
        warm = eng.seq_create(0)
        prompt = rng.integers(1, 32000, T).astype(np.int32)
        eng.forward_prefill_chunk(warm, prompt, 0, want_logits=False)
        seq = eng.seq_create(1)
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        eng.forward_prefill_chunk(seq, prompt, 0, want_logits=False)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        print(f"profiled the prefill of one {T}-token prompt")
        return 0
    B = max(1, min(args.batch, 64))
    model = synth.cached_model(synth.SHAPE_110M, seed=1234)
    eng = NitroEngine(model, EngineConfig(total_blocks=1024, max_new_tokens=100000, max_batch=64,
                                          max_prefill_tokens=256, device=0))
    for i in range(B):
        eng.add_request(i, rng.integers(1, 32000, int(rng.integers(128, 201))).astype(np.int32))
    while True:  # admission, one prefill per step (the reference scheduler's order)
        r = eng.step()
        if len(eng.running_batch()) == B and r.prefill_req_id < 0:
            break
    eng.step()
    eng.replay_decode(3)
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    eng.replay_decode(1)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print(f"profiled one decode step of {B} sequences")
    return 0


if __name__ == "__main__":
    sys.exit(main())
