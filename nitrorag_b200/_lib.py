"""ctypes binding of ``libnitro_engine.so`` (the C ABI in include/nitro_engine.h).

The library is loaded from this package directory only; there is no fallback: a missing
or unloadable library raises ``EngineLibraryMissing``."""
from __future__ import annotations

import ctypes as C
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libnitro_engine.so")

NR_OK = 0
NR_ERR = {
    -1: "NR_ERR_INVALID", -2: "NR_ERR_IO", -3: "NR_ERR_FORMAT", -4: "NR_ERR_CUDA",
    -5: "NR_ERR_NO_BLOCKS", -6: "NR_ERR_NO_DEVICE", -7: "NR_ERR_UNKNOWN_SEQ",
    -8: "NR_ERR_CAPACITY", -9: "NR_ERR_TIMEOUT",
}
KERNEL_CLASSES = ["embed", "qkv", "attention", "wo", "w13", "w2", "logits", "argmax", "attn_merge"]
NR_Q8_FIXED = 0
NR_Q8_FAITHFUL = 1
NR_SCHED_REFERENCE = 0
NR_SCHED_PACKED = 1
NR_KV_F32 = 0
NR_KV_BF16 = 1


class EngineLibraryMissing(RuntimeError):
    pass


class NrConfig(C.Structure):
    _fields_ = [
        ("total_blocks", C.c_int32), ("max_tokens_per_batch", C.c_int32),
        ("max_new_tokens", C.c_int32), ("block_size", C.c_int32), ("sched_mode", C.c_int32),
        ("q8_mode", C.c_int32), ("max_batch", C.c_int32), ("max_prefill_tokens", C.c_int32),
        ("device", C.c_int32), ("kv_dtype", C.c_int32), ("reserved", C.c_int32 * 6),
    ]


class NrStepOut(C.Structure):
    _fields_ = [
        ("n_released", C.c_int32), ("prefill_req_id", C.c_int32), ("prefill_tokens", C.c_int32),
        ("prefill_hits", C.c_int32), ("n_decode", C.c_int32), ("n_emitted", C.c_int32),
        ("emitted_cap", C.c_int32), ("emitted_req_ids", C.POINTER(C.c_int32)),
        ("emitted_tokens", C.POINTER(C.c_int32)), ("emitted_logits", C.POINTER(C.c_float)),
        ("n_prefill", C.c_int32),
    ]


class NrPlan(C.Structure):
    _fields_ = [
        ("n_released", C.c_int32), ("prefill_req_id", C.c_int32), ("prefill_start", C.c_int32),
        ("prefill_tokens", C.c_int32), ("prefill_done", C.c_int32), ("prefill_hits", C.c_int32),
        ("n_decode", C.c_int32), ("decode_cap", C.c_int32), ("decode_req_ids", C.POINTER(C.c_int32)),
        ("n_prefill", C.c_int32), ("prefill_cap", C.c_int32), ("prefill_req_ids", C.POINTER(C.c_int32)),
        ("prefill_starts", C.POINTER(C.c_int32)), ("prefill_lens", C.POINTER(C.c_int32)),
        ("prefill_dones", C.POINTER(C.c_int32)),
    ]


class NrStats(C.Structure):
    _fields_ = [("steps", C.c_int64), ("prefill_tokens", C.c_int64), ("decode_tokens", C.c_int64),
                ("cache_hit_pages", C.c_int64), ("evictions", C.c_int64), ("kernel_launches", C.c_int64)]


P = C.c_void_p
I32 = C.c_int32
PI32 = C.POINTER(C.c_int32)
PF = C.POINTER(C.c_float)
U64 = C.c_uint64

# nr_step_fn of include/nitro_server.h: int (*)(void* ctx, nr_engine*, nr_step_out*)
STEP_FN = C.CFUNCTYPE(C.c_int, P, P, C.POINTER(NrStepOut))

# name -> (restype, argtypes); every symbol declared in include/nitro_engine.h and
# include/nitro_server.h
SIGNATURES = {
    "nr_config_default": (None, [C.POINTER(NrConfig)]),
    "nr_engine_create": (C.c_int, [C.POINTER(NrConfig), C.c_char_p, C.POINTER(P)]),
    "nr_engine_create_from_memory": (C.c_int, [C.POINTER(NrConfig), P, C.c_size_t, C.POINTER(P)]),
    "nr_engine_create_host_only": (C.c_int, [C.POINTER(NrConfig), PI32, C.POINTER(P)]),
    "nr_engine_destroy": (C.c_int, [P]),
    "nr_model_shape": (C.c_int, [P, PI32]),
    "nr_engine_stream": (P, [P]),
    "nr_last_error": (C.c_char_p, [P]),
    "nr_add_request": (C.c_int, [P, I32, PI32, I32]),
    "nr_has_active": (C.c_int, [P]),
    "nr_step": (C.c_int, [P, C.POINTER(NrStepOut)]),
    "nr_step_plan": (C.c_int, [P, C.POINTER(NrPlan)]),
    "nr_step_commit": (C.c_int, [P, C.POINTER(NrPlan), PI32, I32]),
    "nr_request_tokens": (C.c_int, [P, I32, PI32, I32, PI32]),
    "nr_request_state": (C.c_int, [P, I32, PI32]),
    "nr_request_block_table": (C.c_int, [P, I32, PI32, I32, PI32]),
    "nr_running_batch": (C.c_int, [P, PI32, I32, PI32]),
    "nr_seq_create": (C.c_int, [P, I32, PI32]),
    "nr_seq_append": (C.c_int, [P, I32, I32]),
    "nr_seq_flush_cache": (C.c_int, [P, I32]),
    "nr_seq_release": (C.c_int, [P, I32]),
    "nr_seq_destroy": (C.c_int, [P, I32]),
    "nr_seq_block_table": (C.c_int, [P, I32, PI32, I32, PI32]),
    "nr_seq_info": (C.c_int, [P, I32, PI32, C.POINTER(U64)]),
    "nr_forward_prefill": (C.c_int, [P, I32, PI32, I32, I32, PF, PI32]),
    "nr_forward_decode": (C.c_int, [P, I32, PI32, PI32, PI32, PF, PI32]),
    "nr_forward_paged": (C.c_int, [P, I32, I32, I32, PF, PI32]),
    "nr_ingest_prompt": (C.c_int, [P, I32, PI32, I32, I32, PF, PI32, PI32]),
    "nr_pool_free_count": (C.c_int, [P]),
    "nr_pool_free_list": (C.c_int, [P, PI32, I32, PI32]),
    "nr_pool_block_state": (C.c_int, [P, I32, PI32]),
    "nr_cache_lookup": (C.c_int, [P, U64, PI32]),
    "nr_cache_size": (C.c_int, [P]),
    "nr_cache_is_cached": (C.c_int, [P, I32]),
    "nr_cache_lru": (C.c_int, [P, PI32, I32, PI32]),
    "nr_cache_entries": (C.c_int, [P, C.POINTER(U64), PI32, I32, PI32]),
    "nr_pool_read_page": (C.c_int, [P, I32, PF, PF]),
    "nr_hash_block_state": (U64, [U64, PI32, I32]),
    "nr_argmax": (I32, [PF, I32]),
    "nr_engine_stats": (C.c_int, [P, C.POINTER(NrStats)]),
    "nr_engine_set_profiling": (C.c_int, [P, I32]),
    "nr_engine_kernel_times": (C.c_int, [P, C.POINTER(C.c_double), C.POINTER(C.c_int64)]),
    "nr_replay_decode": (C.c_int, [P, I32]),
    "nr_replay_decode_attention": (C.c_int, [P, I32, I32]),
    "nr_decode_last_outputs": (C.c_int, [P, PI32, PF, PI32]),
    "nr_paged_attention_workspace_size": (C.c_size_t, [I32, I32, I32, I32]),
    "nr_paged_attention_decode": (C.c_int, [P, P, P, P, I32, P, I32, I32, I32, I32, I32, I32, P, P, P, P]),
    "nr_paged_attention_decode_static": (C.c_int, [P, P, P, P, I32, P, I32, I32, I32, I32, I32, I32, P, P, P]),
    "nr_q8_matmul": (C.c_int, [P, P, P, P, I32, I32, I32, I32, P]),
    "nr_q8_quantized_size": (C.c_size_t, [C.c_int64]),
    "nr_quantize_q8_device": (C.c_int, [P, C.c_int64, P, P]),
    "nr_quantize_q8": (C.c_int, [P, C.c_int64, P, I32]),
    "nr_quantize_model_file": (C.c_int, [C.c_char_p, C.c_char_p, I32]),
    "nr_server_create": (C.c_int, [P, C.c_char_p, I32, STEP_FN, P, C.POINTER(P)]),
    "nr_server_port": (C.c_int, [P]),
    "nr_server_poll": (C.c_int, [P, I32]),
    "nr_server_run": (C.c_int, [P]),
    "nr_server_stop": (C.c_int, [P]),
    "nr_server_counters": (C.c_int, [P, C.POINTER(C.c_int64)]),
    "nr_server_destroy": (C.c_int, [P]),
}

_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise EngineLibraryMissing(
                f"{LIB_PATH} is not built; run `python -m nitrorag_b200.build` (needs nvcc)")
        try:
            handle = C.CDLL(LIB_PATH)
        except OSError as exc:
            raise EngineLibraryMissing(f"cannot load {LIB_PATH}: {exc}") from exc
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


class NrError(RuntimeError):
    def __init__(self, code: int, where: str, detail: str = ""):
        self.code = code
        super().__init__(f"{where}: {NR_ERR.get(code, code)} {detail}".strip())


def check(code: int, where: str, engine=None) -> int:
    if code < 0:
        detail = ""
        try:
            msg = lib().nr_last_error(engine)
            detail = msg.decode() if msg else ""
        except Exception:  # pragma: no cover - diagnostics only
            pass
        raise NrError(code, where, detail)
    return code
