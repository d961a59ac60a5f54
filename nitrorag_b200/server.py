"""Python face of the NitroRPC front end (include/nitro_server.h): the reference's
Server_Inference loop (src/Server_Inference.cpp) on the engine's C ABI.

    eng = NitroEngine("model.bin", EngineConfig(max_new_tokens=64))
    with NitroServer(eng, port=8081) as srv:
        srv.run()          # engine loop on this thread until srv.stop()

A client sends a little-endian int32 count and that many int32 token ids, then reads one
int32 per generated token until the server closes the connection (``request`` below; the
reference's client is scripts/agent.py:62-70)."""
from __future__ import annotations

import ctypes as C
import socket
import struct

from . import _lib
from ._lib import NrStepOut, lib


def host_step(token_fn):
    """A step function for a host-only engine (nr_step needs a GPU): plan the iteration,
    take the sampled tokens from ``token_fn(engine, plan) -> list[int]`` (one per prompt
    chunk that completes, then one per decode row), commit, and report them like nr_step."""

    def make(engine):
        def step(_ctx, _eng, out):
            try:
                plan = engine.step_plan()
                toks = [int(t) for t in token_fn(engine, plan)]
                engine.step_commit(toks)
            except _lib.NrError as err:
                return err.code
            ids = [c["req_id"] for c in plan["prefills"] if c["done"]] + list(plan["decode_req_ids"])
            o = out.contents
            o.n_released = plan["n_released"]
            o.prefill_req_id = plan["prefill_req_id"]
            o.prefill_tokens = sum(c["tokens"] for c in plan["prefills"])
            o.prefill_hits = plan["prefill_hits"]
            o.n_prefill = len(plan["prefills"])
            o.n_decode = len(plan["decode_req_ids"])
            o.n_emitted = len(toks)
            for i, (rid, tok) in enumerate(zip(ids, toks)):
                if i >= o.emitted_cap:
                    break
                o.emitted_req_ids[i] = rid
                o.emitted_tokens[i] = tok
            return 0

        return _lib.STEP_FN(step)

    return make


class NitroServer:
    def __init__(self, engine, host: str | None = "127.0.0.1", port: int = 0, step=None):
        """step: None for nr_step (a GPU engine), or host_step(...) for a host-only one."""
        self.engine = engine
        self._step_cb = step(engine) if step else _lib.STEP_FN()
        h = C.c_void_p()
        _lib.check(lib().nr_server_create(engine._h, host.encode() if host else None, port, self._step_cb, None,
                                          C.byref(h)), "nr_server_create")
        self._h = h

    @property
    def port(self) -> int:
        return lib().nr_server_port(self._h)

    def poll(self, wait_ms: int = 10) -> int:
        """One engine-loop iteration; returns the number of tokens emitted."""
        return _lib.check(lib().nr_server_poll(self._h, wait_ms), "nr_server_poll", self.engine._h)

    def run(self) -> None:
        _lib.check(lib().nr_server_run(self._h), "nr_server_run", self.engine._h)

    def stop(self) -> None:
        lib().nr_server_stop(self._h)

    def counters(self) -> dict:
        c = (C.c_int64 * 4)()
        _lib.check(lib().nr_server_counters(self._h, c), "nr_server_counters")
        return dict(accepted=c[0], refused=c[1], tokens_sent=c[2], finished=c[3])

    def close(self) -> None:
        if self._h:
            lib().nr_server_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def request(host: str, port: int, prompt, timeout: float = 60.0) -> list[int]:
    """Client side of the wire format: send the prompt, read token ids until the server
    closes the connection."""
    with socket.create_connection((host, port), timeout=timeout) as s:
        s.sendall(struct.pack("<i", len(prompt)) + struct.pack(f"<{len(prompt)}i", *[int(t) for t in prompt]))
        data = b""
        while True:
            chunk = s.recv(65536)
            if not chunk:
                break
            data += chunk
    return list(struct.unpack(f"<{len(data) // 4}i", data[: len(data) // 4 * 4]))
