"""The NitroRPC front end on the GPU: clients send prompts over a localhost socket to a
server whose engine loop runs nr_step on a seeded tiny model; the tokens streamed back
must be the greedy tokens the reference's own Continuous_Scheduler generates for each
prompt (ref_fixed build)."""
import threading

import numpy as np
import pytest

from nitrorag_b200 import EngineConfig, NitroEngine
from nitrorag_b200.server import NitroServer, request

pytestmark = pytest.mark.gpu
MAX_NEW = 8


def _reference_tokens(ref, model, prompt):
    ref.open(model, 256, 64)
    h = ref.new_request(0, prompt)
    ref.sched_add(h)
    while ref.sched_has_active():
        ref.sched_step(MAX_NEW)
    toks = ref.generated(h)
    ref.close()
    return toks


def test_server_streams_reference_tokens(ref_fixed, tiny_model):
    rng = np.random.default_rng(21)
    prompts = [rng.integers(0, 512, n).astype(np.int32).tolist() for n in (37, 5, 120)]
    want = [_reference_tokens(ref_fixed, tiny_model, p) for p in prompts]
    eng = NitroEngine(tiny_model, EngineConfig(total_blocks=64, max_new_tokens=MAX_NEW, max_batch=8,
                                               max_prefill_tokens=256))
    srv = NitroServer(eng, "127.0.0.1", 0)
    got = [None] * len(prompts)

    def client(i):
        got[i] = request("127.0.0.1", srv.port, prompts[i])

    threads = [threading.Thread(target=client, args=(i,)) for i in range(len(prompts))]
    for t in threads:
        t.start()
    for _ in range(5000):
        if all(g is not None for g in got):
            break
        srv.poll(5)
    for t in threads:
        t.join(timeout=30)
    assert got == want
    c = srv.counters()
    assert c["finished"] == 3 and c["tokens_sent"] == 3 * MAX_NEW
    srv.close()
    eng.close()


def test_nitro_server_process(ref_fixed, tiny_model):
    """The server process itself (nitrorag_b200/nitro_server, the reference's
    Server_Inference main): start it on a free port, send one prompt, read the stream,
    stop it with SIGTERM."""
    import os
    import signal
    import subprocess

    from nitrorag_b200 import build
    prompt = np.random.default_rng(22).integers(0, 512, 64).astype(np.int32).tolist()
    want = _reference_tokens(ref_fixed, tiny_model, prompt)
    proc = subprocess.Popen([build.SERVER, tiny_model, "--port", "0", "--host", "127.0.0.1", "--blocks", "64",
                             "--max-new", str(MAX_NEW)], stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
    try:
        line = proc.stdout.readline()
        assert "listening on port" in line, (line, proc.stderr.read() if proc.poll() is not None else "")
        port = int(line.split()[-1])
        assert request("127.0.0.1", port, prompt) == want
    finally:
        proc.send_signal(signal.SIGTERM)
        proc.wait(timeout=30)
    assert proc.returncode == 0
    assert os.path.exists(build.SERVER)
