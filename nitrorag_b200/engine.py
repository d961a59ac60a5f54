"""Python face of the engine, mirroring the reference's engine surface (nvivek17/NitroRAG):

    forward_prefill_chunk   src/model_q8.cpp:424      forward_decode_batch   :571
    forward_paged           src/model_q8.cpp:244      ingest_prompt          :695
    argmax                  src/model_q8.cpp:559      hash_block_state       src/pagedMemory.hpp:14
    Continuous_Scheduler::{add_request, has_active_requests, step}   src/pagedMemory.hpp:310-398
    Sequence::{allocate_next_token, flush_cache, release}            src/pagedMemory.hpp:245-283

Everything runs through the C ABI of libnitro_engine.so; errors raise ``NrError`` instead
of exiting the process as the reference does."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import (NR_KV_BF16, NR_KV_F32, NR_Q8_FAITHFUL, NR_Q8_FIXED, NR_SCHED_PACKED, NR_SCHED_REFERENCE, NrConfig,
                   NrError, NrPlan, NrStats, NrStepOut, check, lib)

__all__ = ["NitroEngine", "EngineConfig", "StepResult", "hash_block_state", "argmax",
           "NR_Q8_FIXED", "NR_Q8_FAITHFUL", "NR_SCHED_REFERENCE", "NR_SCHED_PACKED", "NR_KV_F32", "NR_KV_BF16",
           "NrError", "FNV_OFFSET_BASIS"]

FNV_OFFSET_BASIS = 14695981039346656037


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


def _pi32(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_int32))


def _pf(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.POINTER(C.c_float))


def hash_block_state(parent: int, tokens) -> int:
    t = _i32(tokens)
    return int(lib().nr_hash_block_state(C.c_uint64(parent), _pi32(t), len(t)))


def argmax(x) -> int:
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    return int(lib().nr_argmax(_pf(a), len(a)))


@dataclass
class EngineConfig:
    total_blocks: int = 1000
    max_tokens_per_batch: int = 256
    max_new_tokens: int = 20
    q8_mode: int = NR_Q8_FIXED
    max_batch: int = 256
    max_prefill_tokens: int = 1024
    device: int = 0
    sched_mode: int = 0  # NR_SCHED_REFERENCE; 1 = NR_SCHED_PACKED
    kv_dtype: int = 0    # NR_KV_F32; 1 = NR_KV_BF16 (bf16 K/V pages)

    def to_c(self) -> NrConfig:
        c = NrConfig()
        lib().nr_config_default(C.byref(c))
        c.total_blocks = self.total_blocks
        c.max_tokens_per_batch = self.max_tokens_per_batch
        c.max_new_tokens = self.max_new_tokens
        c.q8_mode = self.q8_mode
        c.max_batch = self.max_batch
        c.max_prefill_tokens = self.max_prefill_tokens
        c.device = self.device
        c.sched_mode = self.sched_mode
        c.kv_dtype = self.kv_dtype
        return c


@dataclass
class StepResult:
    n_released: int
    prefill_req_id: int
    prefill_tokens: int
    prefill_hits: int
    n_decode: int
    emitted: list  # [(req_id, token)]
    logits: np.ndarray | None
    n_prefill: int = 0  # prompt chunks this step (prefill_tokens / prefill_hits are totals)


class NitroEngine:
    """One engine per GPU (or a host-only engine with ``device=-1`` / ``shape=``)."""

    def __init__(self, model_path: str | None = None, config: EngineConfig | None = None,
                 shape: tuple | None = None):
        self.config = config or EngineConfig()
        c = self.config.to_c()
        h = C.c_void_p()
        if shape is not None:
            s = _i32(shape)
            rc = lib().nr_engine_create_host_only(C.byref(c), _pi32(s), C.byref(h))
        else:
            rc = lib().nr_engine_create(C.byref(c), model_path.encode(), C.byref(h))
        if rc < 0:
            msg = lib().nr_last_error(None)
            raise NrError(rc, "nr_engine_create", msg.decode() if msg else "")
        self._h = h
        s = (C.c_int32 * 7)()
        lib().nr_model_shape(self._h, s)
        (self.dim, self.hidden_dim, self.n_layers, self.n_heads, self.n_kv_heads,
         self.vocab_size, self.seq_len) = list(s)
        self.head_dim = self.dim // self.n_heads
        self.kv_dim = self.n_kv_heads * self.head_dim

    # ------------------------------------------------------------ lifecycle
    def close(self):
        if getattr(self, "_h", None):
            lib().nr_engine_destroy(self._h)
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

    def _check(self, rc, where):
        return check(rc, where, self._h)

    @property
    def stream(self) -> int:
        return lib().nr_engine_stream(self._h) or 0

    def stats(self) -> dict:
        s = NrStats()
        self._check(lib().nr_engine_stats(self._h, C.byref(s)), "nr_engine_stats")
        return {k: getattr(s, k) for k, _ in NrStats._fields_}

    def set_profiling(self, enable: bool) -> None:
        self._check(lib().nr_engine_set_profiling(self._h, int(enable)), "nr_engine_set_profiling")

    def kernel_times(self) -> dict:
        """{class: (total_ms, launches)} accumulated since profiling was enabled."""
        ms = (C.c_double * len(_lib.KERNEL_CLASSES))()
        n = (C.c_int64 * len(_lib.KERNEL_CLASSES))()
        self._check(lib().nr_engine_kernel_times(self._h, ms, n), "nr_engine_kernel_times")
        return {name: (ms[i], n[i]) for i, name in enumerate(_lib.KERNEL_CLASSES)}

    def replay_decode(self, n: int) -> None:
        self._check(lib().nr_replay_decode(self._h, n), "nr_replay_decode")

    def replay_decode_attention(self, n: int, with_merge: bool = False) -> None:
        """Enqueue the last decode step's attention launches (all layers) n more times."""
        self._check(lib().nr_replay_decode_attention(self._h, n, int(with_merge)), "nr_replay_decode_attention")

    def last_decode_outputs(self, want_logits: bool = False):
        """(argmax ids, logits or None) of the most recent decode step or replay."""
        cap = self.config.max_batch
        am = np.zeros(cap, np.int32)
        lg = np.zeros((cap, self.vocab_size), np.float32) if want_logits else None
        B = C.c_int32(0)
        self._check(lib().nr_decode_last_outputs(self._h, _pi32(am), _pf(lg), C.byref(B)), "nr_decode_last_outputs")
        return am[:B.value].copy(), (None if lg is None else lg[:B.value].copy())

    # ------------------------------------------------------------ scheduler
    def add_request(self, req_id: int, prompt) -> None:
        p = _i32(prompt)
        self._check(lib().nr_add_request(self._h, req_id, _pi32(p), len(p)), "nr_add_request")

    def has_active_requests(self) -> bool:
        return self._check(lib().nr_has_active(self._h), "nr_has_active") == 1

    def step(self, want_logits: bool = False, cap: int | None = None) -> StepResult:
        cap = cap or (self.config.max_batch + 1)
        ids = np.zeros(cap, np.int32)
        toks = np.zeros(cap, np.int32)
        lg = np.zeros((cap, self.vocab_size), np.float32) if want_logits else None
        out = NrStepOut()
        out.emitted_cap = cap
        out.emitted_req_ids = _pi32(ids)
        out.emitted_tokens = _pi32(toks)
        out.emitted_logits = _pf(lg)
        self._check(lib().nr_step(self._h, C.byref(out)), "nr_step")
        n = out.n_emitted
        return StepResult(out.n_released, out.prefill_req_id, out.prefill_tokens, out.prefill_hits,
                          out.n_decode, list(zip(ids[:n].tolist(), toks[:n].tolist())),
                          None if lg is None else lg[:n].copy(), out.n_prefill)

    def step_plan(self, cap: int = 4096) -> dict:
        ids = np.zeros(cap, np.int32)
        rows = [np.zeros(cap, np.int32) for _ in range(4)]  # req ids, starts, lengths, done flags
        p = NrPlan()
        p.decode_cap = cap
        p.decode_req_ids = _pi32(ids)
        p.prefill_cap = cap
        p.prefill_req_ids, p.prefill_starts, p.prefill_lens, p.prefill_dones = (_pi32(r) for r in rows)
        self._check(lib().nr_step_plan(self._h, C.byref(p)), "nr_step_plan")
        self._plan = p
        self._plan_ids = (ids, rows)
        k = p.n_prefill
        return dict(n_released=p.n_released, prefill_req_id=p.prefill_req_id, prefill_start=p.prefill_start,
                    prefill_tokens=p.prefill_tokens, prefill_done=bool(p.prefill_done),
                    prefill_hits=p.prefill_hits, decode_req_ids=ids[:p.n_decode].tolist(),
                    prefills=[dict(req_id=int(rows[0][i]), start=int(rows[1][i]), tokens=int(rows[2][i]),
                                   done=bool(rows[3][i])) for i in range(k)])

    def step_commit(self, tokens) -> None:
        t = _i32(tokens)
        self._check(lib().nr_step_commit(self._h, C.byref(self._plan), _pi32(t), len(t)), "nr_step_commit")

    def request_tokens(self, req_id: int) -> list:
        return self._read_list(lib().nr_request_tokens, req_id)

    def request_state(self, req_id: int) -> dict:
        f = (C.c_int32 * 4)()
        self._check(lib().nr_request_state(self._h, req_id, f), "nr_request_state")
        return dict(prefill_idx=f[0], is_prefill_done=bool(f[1]), is_finished=bool(f[2]),
                    next_token_to_process=f[3])

    def request_block_table(self, req_id: int) -> list:
        return self._read_list(lib().nr_request_block_table, req_id)

    def running_batch(self) -> list:
        n = C.c_int32()
        self._check(lib().nr_running_batch(self._h, None, 0, C.byref(n)), "nr_running_batch")
        out = np.zeros(max(n.value, 1), np.int32)
        self._check(lib().nr_running_batch(self._h, _pi32(out), n.value, C.byref(n)), "nr_running_batch")
        return out[:n.value].tolist()

    def _read_list(self, fn, key) -> list:
        n = C.c_int32()
        self._check(fn(self._h, key, None, 0, C.byref(n)), fn.__name__)
        out = np.zeros(max(n.value, 1), np.int32)
        self._check(fn(self._h, key, _pi32(out), n.value, C.byref(n)), fn.__name__)
        return out[:n.value].tolist()

    # ------------------------------------------------------------ sequences
    def seq_create(self, seq_id: int = 0) -> int:
        h = C.c_int32()
        self._check(lib().nr_seq_create(self._h, seq_id, C.byref(h)), "nr_seq_create")
        return h.value

    def allocate_next_token(self, seq: int, token: int) -> None:
        self._check(lib().nr_seq_append(self._h, seq, token), "nr_seq_append")

    def flush_cache(self, seq: int) -> None:
        self._check(lib().nr_seq_flush_cache(self._h, seq), "nr_seq_flush_cache")

    def release(self, seq: int) -> None:
        self._check(lib().nr_seq_release(self._h, seq), "nr_seq_release")

    def seq_destroy(self, seq: int) -> None:
        self._check(lib().nr_seq_destroy(self._h, seq), "nr_seq_destroy")

    def block_table(self, seq: int) -> list:
        return self._read_list(lib().nr_seq_block_table, seq)

    def seq_info(self, seq: int) -> dict:
        info = (C.c_int32 * 3)()
        h = C.c_uint64()
        self._check(lib().nr_seq_info(self._h, seq, info, C.byref(h)), "nr_seq_info")
        return dict(logical_token_count=info[0], token_buffer=info[1], n_blocks=info[2], current_hash=h.value)

    # ------------------------------------------------------------ forward passes
    def forward_prefill_chunk(self, seq: int, tokens, start_pos: int, want_logits: bool = True):
        t = _i32(tokens)
        lg = np.zeros(self.vocab_size, np.float32) if want_logits else None
        am = C.c_int32()
        self._check(lib().nr_forward_prefill(self._h, seq, _pi32(t), len(t), start_pos, _pf(lg), C.byref(am)),
                    "nr_forward_prefill")
        return lg, am.value

    def forward_decode_batch(self, tokens, positions, seqs, want_logits: bool = True):
        t, p, s = _i32(tokens), _i32(positions), _i32(seqs)
        B = len(t)
        lg = np.zeros((B, self.vocab_size), np.float32) if want_logits else None
        am = np.zeros(B, np.int32)
        self._check(lib().nr_forward_decode(self._h, B, _pi32(t), _pi32(p), _pi32(s), _pf(lg), _pi32(am)),
                    "nr_forward_decode")
        return lg, am

    def forward_paged(self, seq: int, token: int, pos: int, want_logits: bool = True):
        lg = np.zeros(self.vocab_size, np.float32) if want_logits else None
        am = C.c_int32()
        self._check(lib().nr_forward_paged(self._h, seq, token, pos, _pf(lg), C.byref(am)), "nr_forward_paged")
        return lg, am.value

    def ingest_prompt(self, seq: int, prompt, enable_prefix_caching: bool = True):
        t = _i32(prompt)
        lg = np.zeros(self.vocab_size, np.float32)
        n = C.c_int32()
        comp = C.c_int32()
        self._check(lib().nr_ingest_prompt(self._h, seq, _pi32(t), len(t), int(enable_prefix_caching), _pf(lg),
                                           C.byref(n), C.byref(comp)), "nr_ingest_prompt")
        return n.value, comp.value, (lg if comp.value > 0 else None)

    # ------------------------------------------------------------ pool / cache
    def free_count(self) -> int:
        return self._check(lib().nr_pool_free_count(self._h), "nr_pool_free_count")

    def free_list(self) -> list:
        n = C.c_int32()
        self._check(lib().nr_pool_free_list(self._h, None, 0, C.byref(n)), "nr_pool_free_list")
        out = np.zeros(max(n.value, 1), np.int32)
        self._check(lib().nr_pool_free_list(self._h, _pi32(out), n.value, C.byref(n)), "nr_pool_free_list")
        return out[:n.value].tolist()

    def block_state(self, block: int) -> tuple:
        st = (C.c_int32 * 4)()
        self._check(lib().nr_pool_block_state(self._h, block, st), "nr_pool_block_state")
        return tuple(st)

    def cache_lookup(self, h: int) -> int:
        b = C.c_int32()
        self._check(lib().nr_cache_lookup(self._h, C.c_uint64(h), C.byref(b)), "nr_cache_lookup")
        return b.value

    def cache_size(self) -> int:
        return self._check(lib().nr_cache_size(self._h), "nr_cache_size")

    def is_cached(self, block: int) -> bool:
        return self._check(lib().nr_cache_is_cached(self._h, block), "nr_cache_is_cached") == 1

    def lru(self) -> list:
        n = C.c_int32()
        self._check(lib().nr_cache_lru(self._h, None, 0, C.byref(n)), "nr_cache_lru")
        out = np.zeros(max(n.value, 1), np.int32)
        self._check(lib().nr_cache_lru(self._h, _pi32(out), n.value, C.byref(n)), "nr_cache_lru")
        return out[:n.value].tolist()

    def cache_entries(self) -> dict:
        n = C.c_int32()
        self._check(lib().nr_cache_entries(self._h, None, None, 0, C.byref(n)), "nr_cache_entries")
        hs = np.zeros(max(n.value, 1), np.uint64)
        bs = np.zeros(max(n.value, 1), np.int32)
        self._check(lib().nr_cache_entries(self._h, hs.ctypes.data_as(C.POINTER(C.c_uint64)), _pi32(bs), n.value,
                                           C.byref(n)), "nr_cache_entries")
        return {int(h): int(b) for h, b in zip(hs[:n.value], bs[:n.value])}

    def read_page(self, block: int):
        n = self.n_layers * 16 * self.kv_dim
        k = np.zeros(n, np.float32)
        v = np.zeros(n, np.float32)
        self._check(lib().nr_pool_read_page(self._h, block, _pf(k), _pf(v)), "nr_pool_read_page")
        return k.reshape(self.n_layers, 16, self.kv_dim), v.reshape(self.n_layers, 16, self.kv_dim)
