"""The multi-GPU path is independent replicas (no collective on the data path): each rank
owns its own engine, page pool, prefix cache and 64 requests.  This runs that host-side
logic as two gloo ranks on the CPU: per-rank workloads, each replica's scheduler (host-only
engine), and the only cross-rank steps the benchmark takes (barrier, max of timings)."""
import os
import socket
import sys

import pytest

from conftest import ROOT


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, out_path):
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    import torch
    import torch.distributed as dist

    import bench
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    prompts = bench.prompts_for(rank)
    order, ctx = bench.schedule_contexts(prompts, 3)
    # every replica decodes its own 64 requests: gather the context sums to compare
    t = torch.tensor([float(sum(ctx)), float(len(order)), 1.0 + rank], dtype=torch.float64)
    gathered = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(gathered, t)
    elapsed = torch.tensor([1.0 + rank], dtype=torch.float64)  # stand-in for a device time
    dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
    dist.barrier()
    if rank == 0:
        with open(out_path, "w") as f:
            f.write(repr([g.tolist() for g in gathered]) + "\n" + repr(float(elapsed.item())))
    dist.destroy_process_group()


def test_two_replicas_on_gloo(tmp_path):
    import torch.multiprocessing as mp
    out = str(tmp_path / "res.txt")
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("rank hung")
        assert p.exitcode == 0
    lines = open(out).read().splitlines()
    gathered = eval(lines[0])
    assert float(lines[1]) == 2.0  # max over ranks
    assert gathered[0][1] == gathered[1][1] == 64.0  # each replica runs all 64 of its requests
    assert gathered[0][0] != gathered[1][0]  # ranks draw different workloads (seed 100 + rank)
