"""One decode step of a 64-request batch inside a CUDA profiler range, for capturing
individual kernels with a profiler started as `--profile-from-start off`:

    ncu --profile-from-start off --set full --clock-control none -k regex:tc_gemm -c 1 \\
        -o out python -m nitrorag_b200.profile_step

The case is the benchmark's decode step shape (110M Q8_0 model, 64 sequences) with short
prompts (U[128, 200] tokens) and a 1024-page pool, so the device holds ~1.7 GB: small
enough for multi-pass captures, with weights and K/V still far larger than L2.  The step
runs eagerly (no CUDA graph) so each kernel is an ordinary launch.
"""
from __future__ import annotations

import os
import sys


def main() -> int:
    os.environ.setdefault("NITRO_GRAPHS", "0")
    import numpy as np
    import torch

    from . import EngineConfig, NitroEngine, synth

    model = synth.cached_model(synth.SHAPE_110M, seed=1234)
    eng = NitroEngine(model, EngineConfig(total_blocks=1024, max_new_tokens=100000, max_batch=64,
                                          max_prefill_tokens=256, device=0))
    rng = np.random.default_rng(3)
    for i in range(64):
        eng.add_request(i, rng.integers(1, 32000, int(rng.integers(128, 201))).astype(np.int32))
    while True:  # admission, one prefill per step (the reference scheduler's order)
        r = eng.step()
        if len(eng.running_batch()) == 64 and r.prefill_req_id < 0:
            break
    eng.step()
    eng.replay_decode(3)
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    eng.replay_decode(1)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print("profiled one decode step of 64 sequences")
    return 0


if __name__ == "__main__":
    sys.exit(main())
