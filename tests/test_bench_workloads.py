"""The benchmark's decode64 workload: the reference arm takes its decode contexts from the
reference's own Continuous_Scheduler (bench.schedule_contexts, on a narrow model with the
same vocabulary, sequence length and token budget); the engine arm takes them from its own
scheduler.  Both must put the same requests in the same order at the same positions."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def _engine_contexts(prompts, extra_steps):
    from nitrorag_b200 import EngineConfig, NitroEngine
    eng = NitroEngine(config=EngineConfig(total_blocks=8192, max_new_tokens=100000, device=-1),
                      shape=(768, 2048, 12, 12, 12, 32000, 1024))
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
    ctx = [len(prompts[r]) + len(eng.request_tokens(r)) - 1 for r in order]
    eng.close()
    return order, ctx


@pytest.mark.parametrize("rank,world,extra", [(0, 1, 25), (3, 4, 0)])
def test_decode64_contexts_reference_scheduler(rank, world, extra):
    import oracle
    if not oracle.reference_available("fixed"):
        pytest.skip("reference build absent")
    import bench
    prompts = bench.prompts_for(rank, world)
    assert len(prompts) == 64
    want = _engine_contexts(prompts, extra)
    got = bench.schedule_contexts(prompts, extra)
    assert got == want
