"""B200 engine for the Q8_0 prefill/decode step of NitroRAG's inference server.

The product is ``libnitro_engine.so`` (C ABI in ``include/nitro_engine.h``); this package
is its Python face (``engine.NitroEngine``), the build recipe and the seeded synthetic
model/workload generators.  Importing the package does not require a GPU; creating a
GPU engine does, and fails loudly when the library or the device is missing."""
from .engine import (FNV_OFFSET_BASIS, NR_KV_BF16, NR_KV_F32, NR_Q8_FAITHFUL, NR_Q8_FIXED, NR_SCHED_PACKED,
                     NR_SCHED_REFERENCE, EngineConfig, NitroEngine, NrError, StepResult, argmax, hash_block_state)
from .quantize import quantize_model_file, quantize_q8, quantized_size

__all__ = ["NitroEngine", "EngineConfig", "StepResult", "NrError", "hash_block_state", "argmax",
           "NR_Q8_FIXED", "NR_Q8_FAITHFUL", "NR_SCHED_REFERENCE", "NR_SCHED_PACKED", "NR_KV_F32", "NR_KV_BF16",
           "FNV_OFFSET_BASIS", "quantize_q8", "quantize_model_file", "quantized_size"]
