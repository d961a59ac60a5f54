"""The NitroRPC front end (include/nitro_server.h) on a host-only engine: the wire format
of src/NitroRPC.hpp:39-56 over a localhost socket, several concurrent clients streamed
token by token, connections closed when a request finishes, malformed requests refused,
and a client that goes away early not disturbing the others.  Tokens come from a
deterministic stand-in sampler (a host-only engine has no GPU to run nr_step)."""
import socket
import struct
import threading

import pytest

from nitrorag_b200 import EngineConfig, NitroEngine
from nitrorag_b200.server import NitroServer, host_step, request

TINY_SHAPE = (128, 256, 2, 2, 2, 512, 512)
MAX_NEW = 6


def _tokens(engine, plan):
    # token of request r at its g-th generated position: (31 r + 7 g + 1) mod 512
    out = []
    rows = [c["req_id"] for c in plan["prefills"] if c["done"]] + list(plan["decode_req_ids"])
    for r in rows:
        g = len(engine.request_tokens(r))
        out.append((31 * r + 7 * g + 1) % 512)
    return out


def _serve_until(srv, done, limit=2000):
    for _ in range(limit):
        if done():
            return
        srv.poll(5)
    raise AssertionError("server did not finish the requests")


@pytest.fixture
def served():
    eng = NitroEngine(config=EngineConfig(total_blocks=128, max_new_tokens=MAX_NEW, device=-1), shape=TINY_SHAPE)
    srv = NitroServer(eng, "127.0.0.1", 0, step=host_step(_tokens))
    yield eng, srv
    srv.close()
    eng.close()


def test_concurrent_clients_stream_every_token(served):
    eng, srv = served
    shared = list(range(10, 42))
    prompts = [shared + [5, 6, 7], list(range(100, 140)), shared + [9], [3] * 70]
    results = [None] * len(prompts)

    def client(i):
        results[i] = request("127.0.0.1", srv.port, prompts[i])

    threads = [threading.Thread(target=client, args=(i,)) for i in range(len(prompts))]
    for t in threads:
        t.start()
    _serve_until(srv, lambda: all(r is not None for r in results))
    for t in threads:
        t.join(timeout=30)
    # every client got MAX_NEW tokens, exactly its request's generated tokens
    by_prompt = {}
    for rid in range(len(prompts)):
        by_prompt[rid] = eng.request_tokens(rid)
    assert sorted(map(tuple, results)) == sorted(tuple(t) for t in by_prompt.values())
    assert all(len(r) == MAX_NEW for r in results)
    c = srv.counters()
    assert c["accepted"] == 4 and c["refused"] == 0 and c["finished"] == 4 and c["tokens_sent"] == 4 * MAX_NEW


def _raw(port, payload):
    """Bytes the server answers before closing (a reset also counts as closed)."""
    with socket.create_connection(("127.0.0.1", port), timeout=10) as s:
        try:
            s.sendall(payload)
            s.shutdown(socket.SHUT_WR)
            return s.recv(64)
        except ConnectionResetError:
            return b""


@pytest.mark.parametrize("payload", [struct.pack("<i", 0), struct.pack("<i", -3),
                                     struct.pack("<i", 600) + b"\0" * 2400,
                                     struct.pack("<2i", 1, 512),
                                     struct.pack("<i", 4) + b"\1\0\0\0"],
                         ids=["empty", "negative-length", "longer-than-seq-len", "id-outside-vocab", "truncated"])
def test_malformed_requests_are_refused(served, payload):
    eng, srv = served
    got = []
    t = threading.Thread(target=lambda: got.append(_raw(srv.port, payload)))
    t.start()
    t.join(timeout=20)
    assert got == [b""]  # closed without a token
    srv.poll(1)
    assert srv.counters()["refused"] == 1
    assert not eng.has_active_requests()


def test_client_leaving_early_does_not_stop_others(served):
    eng, srv = served
    # client A sends a request and closes immediately
    a = socket.create_connection(("127.0.0.1", srv.port), timeout=10)
    a.sendall(struct.pack("<i", 20) + struct.pack("<20i", *range(20)))
    a.close()
    result = []
    t = threading.Thread(target=lambda: result.append(request("127.0.0.1", srv.port, list(range(50, 90)))))
    t.start()
    _serve_until(srv, lambda: bool(result) and not eng.has_active_requests())
    t.join(timeout=30)
    assert len(result[0]) == MAX_NEW
    assert srv.counters()["finished"] == 2  # the abandoned request ran to completion too


def test_server_executable_is_built():
    """nitrorag_b200/nitro_server links against the library and prints its usage."""
    import subprocess

    from nitrorag_b200 import build
    r = subprocess.run([build.SERVER], capture_output=True, text=True, timeout=30)
    assert r.returncode == 2 and "usage" in r.stderr
