"""Test infrastructure only: ctypes access to the CPU checkers built by oracle/Makefile.

* ``Restatement``   liboracle.so, our scalar restatement of the reference arithmetic
  (nitro_oracle.cpp; every function cites the reference lines it follows).
* ``Reference``     oracle/_ref/libref_{faithful,fixed}.so, the reference's own
  src/model_q8.cpp + src/pagedMemory.hpp behind ref_harness.cpp.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this module; the
engine never does."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = {"faithful": os.path.join(HERE, "_ref", "libref_faithful.so"),
          "fixed": os.path.join(HERE, "_ref", "libref_fixed.so")}

PI32 = C.POINTER(C.c_int32)
PF = C.POINTER(C.c_float)
PU8 = C.POINTER(C.c_uint8)
PU64 = C.POINTER(C.c_uint64)


def _i32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


def _f32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _p(a, t):
    return None if a is None else a.ctypes.data_as(t)


def reference_dir():
    """The reference checkout (nvivek17/NitroRAG): NITRO_REFERENCE_DIR if set, else a
    directory named ``reference`` beside this repository; None where neither holds its
    sources (the GPU hosts, which use the libraries built beforehand)."""
    d = os.environ.get("NITRO_REFERENCE_DIR") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
    return d if os.path.isdir(os.path.join(d, "src")) else None


def build(quiet: bool = True) -> None:
    """Run oracle/Makefile (the reference builds only where its sources exist)."""
    import subprocess
    args = ["oracle"]
    ref = reference_dir()
    if ref:
        args += ["ref", f"REF_SRC={os.path.join(ref, 'src')}"]
    subprocess.run(["make", "-C", HERE, *args], check=True,
                   stdout=subprocess.DEVNULL if quiet else None)


def reference_available(kind: str = "fixed") -> bool:
    return os.path.exists(REF_SO[kind])


class Restatement:
    def __init__(self):
        if not os.path.exists(ORACLE_SO):
            build()
        L = C.CDLL(ORACLE_SO)
        L.orc_quantize_q8.argtypes = [PF, C.c_int64, PU8]
        L.orc_q8_matmul.argtypes = [PF, PF, PU8, C.c_int, C.c_int, C.c_int, C.c_int]
        L.orc_f32_matmul.argtypes = [PF, PF, PF, C.c_int, C.c_int, C.c_int]
        L.orc_rms_norm.argtypes = [PF, PF, PF, C.c_int]
        L.orc_softmax.argtypes = [PF, C.c_int]
        L.orc_argmax.argtypes = [PF, C.c_int]
        L.orc_argmax.restype = C.c_int
        L.orc_fnv_block_hash.argtypes = [C.c_uint64, PI32, C.c_int]
        L.orc_fnv_block_hash.restype = C.c_uint64
        L.orc_rope.argtypes = [PF, PF, C.c_int, C.c_int, C.c_int, C.c_int, PF, PF]
        L.orc_paged_decode_attention.argtypes = [PF, PF, PF, PF, C.c_int64, C.c_int64, PI32, C.c_int, PI32,
                                                 C.c_int, C.c_int, C.c_int, C.c_int]
        L.orc_paged_prefill_attention.argtypes = [PF, PF, PF, PF, C.c_int64, C.c_int64, PI32, C.c_int, C.c_int,
                                                  C.c_int, C.c_int, C.c_int]
        L.orc_model_open.argtypes = [C.c_char_p, C.c_int]
        L.orc_model_open.restype = C.c_void_p
        L.orc_model_close.argtypes = [C.c_void_p]
        L.orc_model_page.argtypes = [C.c_void_p, C.c_int, PF, PF]
        L.orc_model_set_kv_bf16.argtypes = [C.c_void_p, C.c_int]
        L.orc_forward_prefill.argtypes = [C.c_void_p, PI32, PI32, C.c_int, C.c_int, PF, C.c_int]
        L.orc_forward_decode.argtypes = [C.c_void_p, PI32, C.c_int, C.c_int, PI32, PI32, PF, C.c_int]
        self.L = L

    # kernels
    def quantize_q8(self, w) -> bytes:
        w = _f32(w).ravel()
        rem = len(w) % 32
        out = np.zeros(len(w) // 32 * 36 + (4 + rem if rem else 0), np.uint8)
        self.L.orc_quantize_q8(_p(w, PF), len(w), _p(out, PU8))
        return out.tobytes()

    def q8_matmul(self, x, w_aos: bytes, n: int, d: int, last_block_only: bool = False):
        x = _f32(x).reshape(-1, n)
        w = np.frombuffer(w_aos, np.uint8).copy()
        out = np.zeros((x.shape[0], d), np.float32)
        self.L.orc_q8_matmul(_p(out, PF), _p(x, PF), _p(w, PU8), x.shape[0], n, d, int(last_block_only))
        return out

    def f32_matmul(self, x, w, n: int, d: int):
        x = _f32(x).reshape(-1, n)
        w = _f32(w)
        out = np.zeros((x.shape[0], d), np.float32)
        self.L.orc_f32_matmul(_p(out, PF), _p(x, PF), _p(w, PF), x.shape[0], n, d)
        return out

    def rms_norm(self, x, g):
        x, g = _f32(x), _f32(g)
        out = np.zeros_like(x)
        self.L.orc_rms_norm(_p(out, PF), _p(x, PF), _p(g, PF), len(x))
        return out

    def softmax(self, x):
        x = _f32(x).copy()
        self.L.orc_softmax(_p(x, PF), len(x))
        return x

    def argmax(self, x) -> int:
        x = _f32(x)
        return int(self.L.orc_argmax(_p(x, PF), len(x)))

    def hash(self, parent: int, tokens) -> int:
        t = _i32(tokens)
        return int(self.L.orc_fnv_block_hash(C.c_uint64(parent), _p(t, PI32), len(t)))

    def paged_decode_attention(self, q, kpool, vpool, page_stride, layer_off, bt, ctx, n_heads, n_kv_heads, head):
        """Pools in the reference layout (page p, row r at p*page_stride + layer_off + r*kv_dim)."""
        q, kpool, vpool = _f32(q), _f32(kpool), _f32(vpool)
        bt, ctx = _i32(bt), _i32(ctx)
        B = len(ctx)
        out = np.zeros((B, n_heads * head), np.float32)
        self.L.orc_paged_decode_attention(_p(out, PF), _p(q, PF), _p(kpool, PF), _p(vpool, PF), page_stride,
                                          layer_off, _p(bt, PI32), bt.shape[1], _p(ctx, PI32), B, n_heads,
                                          n_kv_heads, head)
        return out

    def paged_prefill_attention(self, q, kpool, vpool, page_stride, layer_off, bt, T, start_pos, n_heads,
                                n_kv_heads, head):
        q, kpool, vpool, bt = _f32(q), _f32(kpool), _f32(vpool), _i32(bt)
        out = np.zeros((T, n_heads * head), np.float32)
        self.L.orc_paged_prefill_attention(_p(out, PF), _p(q, PF), _p(kpool, PF), _p(vpool, PF), page_stride,
                                           layer_off, _p(bt, PI32), T, start_pos, n_heads, n_kv_heads, head)
        return out

    # whole model
    def model(self, path: str, total_pages: int):
        return RestatedModel(self, path, total_pages)


class RestatedModel:
    def __init__(self, o: Restatement, path: str, total_pages: int):
        self.o = o
        self.h = o.L.orc_model_open(path.encode(), total_pages)
        if not self.h:
            raise RuntimeError(f"orc_model_open failed for {path}")
        with open(path, "rb") as f:
            hdr = np.frombuffer(f.read(28), np.int32)
        self.dim, self.hidden, self.n_layers, self.n_heads, self.n_kv_heads, self.vocab, self.seq_len = map(int, hdr)
        self.kv_dim = self.n_kv_heads * (self.dim // self.n_heads)

    def set_kv_bf16(self, on: bool = True):
        """Round K/V to bf16 as they are appended to the pages (the engine's NR_KV_BF16)."""
        self.o.L.orc_model_set_kv_bf16(self.h, int(on))

    def close(self):
        if self.h:
            self.o.L.orc_model_close(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def forward_prefill(self, block_table, tokens, start_pos, last_block_only=False):
        bt, t = _i32(block_table), _i32(tokens)
        lg = np.zeros(self.vocab, np.float32)
        rc = self.o.L.orc_forward_prefill(self.h, _p(bt, PI32), _p(t, PI32), len(t), start_pos, _p(lg, PF),
                                          int(last_block_only))
        assert rc == 0
        return lg

    def forward_decode(self, block_tables, tokens, positions, last_block_only=False):
        """block_tables: list of per-row block lists (padded internally)."""
        B = len(tokens)
        mp = max(len(b) for b in block_tables)
        bt = np.zeros((B, mp), np.int32)
        for i, b in enumerate(block_tables):
            bt[i, :len(b)] = b
        t, p = _i32(tokens), _i32(positions)
        lg = np.zeros((B, self.vocab), np.float32)
        rc = self.o.L.orc_forward_decode(self.h, _p(bt, PI32), mp, B, _p(t, PI32), _p(p, PI32), _p(lg, PF),
                                         int(last_block_only))
        assert rc == 0
        return lg

    def page(self, block):
        n = self.n_layers * 16 * self.kv_dim
        k = np.zeros(n, np.float32)
        v = np.zeros(n, np.float32)
        self.o.L.orc_model_page(self.h, block, _p(k, PF), _p(v, PF))
        return k.reshape(self.n_layers, 16, self.kv_dim), v.reshape(self.n_layers, 16, self.kv_dim)


class Reference:
    """The reference's own code (one instance per process per build: the harness is global)."""

    def __init__(self, kind: str = "fixed"):
        path = REF_SO[kind]
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} not built (needs the reference sources)")
        L = C.CDLL(path)
        sig = {
            "ref_is_fixed": (C.c_int, []), "ref_set_threads": (None, [C.c_int]), "ref_num_procs": (C.c_int, []),
            "ref_close": (None, []), "ref_pool_only": (C.c_int, [C.c_int, C.c_int, C.c_int]),
            "ref_open": (C.c_int, [C.c_char_p, C.c_int, C.c_int]), "ref_config": (C.c_int, [PI32]),
            "ref_req_new": (C.c_int, [C.c_int, PI32, C.c_int]), "ref_seq_alloc_token": (C.c_int, [C.c_int, C.c_int]),
            "ref_seq_flush": (C.c_int, [C.c_int]), "ref_seq_release": (C.c_int, [C.c_int]),
            "ref_seq_info": (C.c_int, [C.c_int, PI32, PU64]),
            "ref_seq_block_table": (C.c_int, [C.c_int, PI32, C.c_int]),
            "ref_free_count": (C.c_int, []), "ref_free_list": (C.c_int, [PI32, C.c_int]),
            "ref_block_state": (C.c_int, [C.c_int, PI32]), "ref_cache_lookup": (C.c_int, [C.c_uint64]),
            "ref_cache_size": (C.c_int, []), "ref_is_cached": (C.c_int, [C.c_int]),
            "ref_cache_entries": (C.c_int, [PU64, PI32, C.c_int]),
            "ref_reverse_entries": (C.c_int, [PI32, PU64, C.c_int]), "ref_lru": (C.c_int, [PI32, C.c_int]),
            "ref_inc_ref": (C.c_int, [C.c_int]), "ref_free_block": (C.c_int, [C.c_int]),
            "ref_allocate_block": (C.c_int, []), "ref_kv_page": (C.c_int, [C.c_int, PF, PF]),
            "ref_kv_fill": (C.c_int, [C.c_float]),
            "ref_hash_block_state": (C.c_uint64, [C.c_uint64, PI32, C.c_int]), "ref_argmax": (C.c_int, [PF, C.c_int]),
            "ref_matmul_bulk_q8": (None, [PF, PF, C.c_void_p, C.c_int, C.c_int, C.c_int]),
            "ref_matmul_q8": (None, [PF, PF, C.c_void_p, C.c_int, C.c_int]),
            "ref_matmul_bulk_f32": (None, [PF, PF, PF, C.c_int, C.c_int, C.c_int]),
            "ref_rms_norm": (None, [PF, PF, PF, C.c_int]), "ref_softmax": (None, [PF, C.c_int]),
            "ref_forward_prefill": (C.c_int, [C.c_int, PI32, C.c_int, C.c_int, PF]),
            "ref_forward_decode": (C.c_int, [C.c_int, PI32, PI32, PI32, PF]),
            "ref_forward_paged": (C.c_int, [C.c_int, C.c_int, C.c_int, PF]),
            "ref_ingest_prompt": (C.c_int, [C.c_int, PI32, C.c_int, C.c_int, PF, PI32]),
            "ref_sched_reset": (C.c_int, []), "ref_sched_add": (C.c_int, [C.c_int]),
            "ref_sched_has_active": (C.c_int, []), "ref_sched_step": (C.c_int, [C.c_int]),
            "ref_sched_decode_logits": (C.c_int, [PF, C.c_int]), "ref_sched_running": (C.c_int, [PI32, C.c_int]),
            "ref_sched_waiting": (C.c_int, []), "ref_req_generated": (C.c_int, [C.c_int, PI32, C.c_int]),
            "ref_req_flags": (C.c_int, [C.c_int, PI32]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        self.L = L
        self.kind = kind
        self.vocab = None

    # setup
    def set_threads(self, n: int):
        self.L.ref_set_threads(n)

    def open(self, path: str, max_tokens: int, total_blocks: int):
        rc = self.L.ref_open(path.encode(), max_tokens, total_blocks)
        assert rc == 0, rc
        cfg = np.zeros(7, np.int32)
        self.L.ref_config(_p(cfg, PI32))
        self.dim, self.hidden, self.n_layers, self.n_heads, self.n_kv_heads, self.vocab, self.seq_len = map(int, cfg)
        self.kv_dim = self.n_kv_heads * (self.dim // self.n_heads)

    def pool_only(self, total_blocks: int, n_layers: int = 1, kv_dim: int = 16):
        assert self.L.ref_pool_only(total_blocks, n_layers, kv_dim) == 0

    def close(self):
        self.L.ref_close()

    # requests / sequences
    def new_request(self, req_id: int, prompt=()) -> int:
        p = _i32(prompt if len(prompt) else [0])
        return self.L.ref_req_new(req_id, _p(p, PI32), len(prompt))

    def alloc_token(self, h: int, token: int):
        assert self.L.ref_seq_alloc_token(h, token) == 0

    def flush(self, h: int):
        self.L.ref_seq_flush(h)

    def release(self, h: int):
        self.L.ref_seq_release(h)

    def seq_info(self, h: int) -> dict:
        out = np.zeros(3, np.int32)
        hh = C.c_uint64()
        self.L.ref_seq_info(h, _p(out, PI32), C.byref(hh))
        return dict(logical_token_count=int(out[0]), token_buffer=int(out[1]), n_blocks=int(out[2]),
                    current_hash=hh.value)

    def block_table(self, h: int) -> list:
        n = self.L.ref_seq_block_table(h, None, 0)
        out = np.zeros(max(n, 1), np.int32)
        self.L.ref_seq_block_table(h, _p(out, PI32), n)
        return out[:n].tolist()

    # pool / cache state
    def free_count(self) -> int:
        return self.L.ref_free_count()

    def free_list(self) -> list:
        n = self.L.ref_free_list(None, 0)
        out = np.zeros(max(n, 1), np.int32)
        self.L.ref_free_list(_p(out, PI32), n)
        return out[:n].tolist()

    def block_state(self, i: int) -> tuple:
        out = np.zeros(4, np.int32)
        self.L.ref_block_state(i, _p(out, PI32))
        return tuple(int(v) for v in out)

    def cache_lookup(self, h: int) -> int:
        return self.L.ref_cache_lookup(C.c_uint64(h))

    def cache_entries(self) -> dict:
        n = self.L.ref_cache_entries(None, None, 0)
        hs = np.zeros(max(n, 1), np.uint64)
        bs = np.zeros(max(n, 1), np.int32)
        self.L.ref_cache_entries(_p(hs, PU64), _p(bs, PI32), n)
        return {int(h): int(b) for h, b in zip(hs[:n], bs[:n])}

    def is_cached(self, i: int) -> bool:
        return self.L.ref_is_cached(i) == 1

    def lru(self) -> list:
        n = self.L.ref_lru(None, 0)
        out = np.zeros(max(n, 1), np.int32)
        self.L.ref_lru(_p(out, PI32), n)
        return out[:n].tolist()

    def kv_page(self, block: int):
        n = self.n_layers * 16 * self.kv_dim
        k = np.zeros(n, np.float32)
        v = np.zeros(n, np.float32)
        self.L.ref_kv_page(block, _p(k, PF), _p(v, PF))
        return k.reshape(self.n_layers, 16, self.kv_dim), v.reshape(self.n_layers, 16, self.kv_dim)

    def hash(self, parent: int, tokens) -> int:
        t = _i32(tokens)
        return int(self.L.ref_hash_block_state(C.c_uint64(parent), _p(t, PI32), len(t)))

    def argmax(self, x) -> int:
        x = _f32(x).copy()
        return int(self.L.ref_argmax(_p(x, PF), len(x)))

    # kernels
    def matmul_bulk_q8(self, x, w_aos: bytes, n: int, d: int):
        x = _f32(x).reshape(-1, n).copy()
        w = np.frombuffer(w_aos, np.uint8).copy()
        out = np.zeros((x.shape[0], d), np.float32)
        self.L.ref_matmul_bulk_q8(_p(out, PF), _p(x, PF), w.ctypes.data, x.shape[0], n, d)
        return out

    def matmul_q8(self, x, w_aos: bytes, n: int, d: int):
        x = _f32(x).ravel().copy()
        w = np.frombuffer(w_aos, np.uint8).copy()
        out = np.zeros(d, np.float32)
        self.L.ref_matmul_q8(_p(out, PF), _p(x, PF), w.ctypes.data, n, d)
        return out

    def matmul_bulk_f32(self, x, w, n: int, d: int):
        x = _f32(x).reshape(-1, n).copy()
        w = _f32(w).copy()
        out = np.zeros((x.shape[0], d), np.float32)
        self.L.ref_matmul_bulk_f32(_p(out, PF), _p(x, PF), _p(w, PF), x.shape[0], n, d)
        return out

    def rms_norm(self, x, g):
        x, g = _f32(x).copy(), _f32(g).copy()
        out = np.zeros_like(x)
        self.L.ref_rms_norm(_p(out, PF), _p(x, PF), _p(g, PF), len(x))
        return out

    def softmax(self, x):
        x = _f32(x).copy()
        self.L.ref_softmax(_p(x, PF), len(x))
        return x

    # forward passes
    def forward_prefill(self, h: int, tokens, start_pos: int):
        t = _i32(tokens)
        lg = np.zeros(self.vocab, np.float32)
        assert self.L.ref_forward_prefill(h, _p(t, PI32), len(t), start_pos, _p(lg, PF)) == 0
        return lg

    def forward_decode(self, tokens, positions, handles):
        t, p, hs = _i32(tokens), _i32(positions), _i32(handles)
        lg = np.zeros((len(t), self.vocab), np.float32)
        assert self.L.ref_forward_decode(len(t), _p(t, PI32), _p(p, PI32), _p(hs, PI32), _p(lg, PF)) == 0
        return lg

    def forward_paged(self, h: int, token: int, pos: int):
        lg = np.zeros(self.vocab, np.float32)
        assert self.L.ref_forward_paged(h, token, pos, _p(lg, PF)) == 0
        return lg

    def ingest_prompt(self, h: int, prompt, enable_cache: bool):
        t = _i32(prompt)
        lg = np.zeros(self.vocab, np.float32)
        n = self.L.ref_ingest_prompt(h, _p(t, PI32), len(t), int(enable_cache), _p(lg, PF), None)
        return n, lg

    # scheduler
    def sched_reset(self):
        self.L.ref_sched_reset()

    def sched_add(self, h: int):
        assert self.L.ref_sched_add(h) == 0

    def sched_has_active(self) -> bool:
        return self.L.ref_sched_has_active() == 1

    def sched_step(self, max_new: int) -> int:
        return self.L.ref_sched_step(max_new)

    def sched_decode_logits(self, rows: int):
        lg = np.zeros((rows, self.vocab), np.float32)
        self.L.ref_sched_decode_logits(_p(lg, PF), rows)
        return lg

    def sched_running(self) -> list:
        n = self.L.ref_sched_running(None, 0)
        out = np.zeros(max(n, 1), np.int32)
        self.L.ref_sched_running(_p(out, PI32), n)
        return out[:n].tolist()

    def generated(self, h: int) -> list:
        n = self.L.ref_req_generated(h, None, 0)
        out = np.zeros(max(n, 1), np.int32)
        self.L.ref_req_generated(h, _p(out, PI32), n)
        return out[:n].tolist()

    def req_flags(self, h: int) -> dict:
        out = np.zeros(4, np.int32)
        self.L.ref_req_flags(h, _p(out, PI32))
        return dict(prefill_idx=int(out[0]), is_prefill_done=bool(out[1]), is_finished=bool(out[2]),
                    next_token_to_process=int(out[3]))
