"""The multi-GPU path is independent replicas (no collective on the data path): request i
of one arrival-ordered stream goes to replica i mod N (nitrorag_b200.replicas), and each
replica owns its engine, page pool and prefix cache.  Here two gloo ranks on the CPU each
serve their part of a Poisson stream with shared prefixes through a host-only engine, in
lockstep with the reference's own Continuous_Scheduler replaying the same part (block
tables, running batch and free list bit-exact every step, the reference's greedy tokens
fed to the engine); rank 0 then checks that the parts cover the stream exactly once.  The
only cross-rank steps are the ones the benchmark takes: gathering counts and the max of
timings."""
import os
import socket
import sys

import pytest

from conftest import ROOT

MAX_NEW = 8
SHAPE = (128, 256, 2, 2, 2, 512, 512)  # synth.SHAPE_TINY


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _serve_part(rank, world, model_path):
    """Replay replica `rank`'s part through the host-only engine and the reference."""
    import oracle
    from nitrorag_b200 import EngineConfig, NitroEngine, replicas, synth
    arrive, prompts = synth.poisson_prefix_workload(n=15, rate=40.0, shared_len=48, lo=8, hi=96, vocab=512, seed=9)
    ids = replicas.partition(len(prompts), world, rank)
    ref = oracle.Reference("fixed")
    ref.set_threads(1)
    ref.open(model_path, 256, 256)
    ref.sched_reset()
    eng = NitroEngine(config=EngineConfig(total_blocks=256, max_new_tokens=MAX_NEW, device=-1), shape=SHAPE)
    handles = {}

    def admit(i):
        handles[i] = ref.new_request(i, prompts[i])
        ref.sched_add(handles[i])

    def tokens(plan):
        ref.sched_step(MAX_NEW)
        out = [ref.generated(handles[c["req_id"]])[-1] for c in plan["prefills"] if c["done"]]
        out += [ref.generated(handles[r])[-1] for r in plan["decode_req_ids"]]
        return out

    def check(k, plan):
        assert eng.running_batch() == ref.sched_running(), (rank, k)
        for i, h in handles.items():
            assert eng.request_block_table(i) == ref.block_table(h), (rank, k, i)
            assert eng.request_tokens(i) == ref.generated(h), (rank, k, i)
        assert eng.free_list() == ref.free_list(), (rank, k)

    res = replicas.run_stream(eng, arrive, prompts, ids, host_tokens=tokens, on_step=check, on_admit=admit)
    assert not ref.sched_has_active()
    eng.close()
    ref.close()
    return ids, res


def _rank_main(rank, world, port, model_path, out_path):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    ids, res = _serve_part(rank, world, model_path)
    parts = [None] * world
    dist.all_gather_object(parts, (rank, ids, {i: len(t) for i, t in res.tokens.items()}, res.prefill_hits))
    elapsed = torch.tensor([1.0 + rank], dtype=torch.float64)  # stand-in for a device time
    dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
    dist.barrier()
    if rank == 0:
        with open(out_path, "w") as f:
            f.write(repr(parts) + "\n" + repr(float(elapsed.item())))
    dist.destroy_process_group()


def test_partition_round_robin():
    from nitrorag_b200 import replicas
    assert replicas.partition(10, 3, 0) == [0, 3, 6, 9]
    assert replicas.partition(10, 3, 2) == [2, 5, 8]
    assert sorted(sum((replicas.partition(50, 8, r) for r in range(8)), [])) == list(range(50))
    with pytest.raises(ValueError):
        replicas.partition(10, 2, 2)


def test_two_replicas_on_gloo(tmp_path):
    import oracle
    if not oracle.reference_available("fixed"):
        pytest.skip("reference build absent")
    import torch.multiprocessing as mp

    from nitrorag_b200 import synth
    model = synth.write_model(str(tmp_path / "tiny.bin"), synth.ModelShape(*SHAPE), seed=11)
    out = str(tmp_path / "res.txt")
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, model, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("rank hung")
        assert p.exitcode == 0
    lines = open(out).read().splitlines()
    parts = eval(lines[0])
    assert float(lines[1]) == 2.0  # max over ranks
    served = sorted(i for _, ids, _, _ in parts for i in ids)
    assert served == list(range(15))  # every request served by exactly one replica
    for rank, ids, counts, _ in parts:
        assert ids == list(range(rank, 15, world))
        assert all(counts[i] == MAX_NEW for i in ids)
    assert all(hits > 0 for _, _, _, hits in parts)  # each replica's own prefix cache is hit
