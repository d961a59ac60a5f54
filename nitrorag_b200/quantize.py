"""Q8_0 quantizer on the GPU through the C ABI: scripts/quantize.py (nvivek17/NitroRAG),
byte for byte.

``quantize_q8(weights)`` is the script's ``quantize_q8`` (quantize.py:7-23): a flat float32
array in, the Q8_0 bytes out (per 32 weights, the last block possibly shorter: the fp32
scale, then the int8 values).  ``quantize_model_file(in, out)`` is the script's driver
(quantize.py:27-60) for a llama2.c-format fp32 checkpoint.  Both run on a GPU and raise
``NrError`` when none is present; there is no CPU path."""
from __future__ import annotations

import numpy as np

from ._lib import check, lib


def quantized_size(n: int) -> int:
    """Bytes of the Q8_0 encoding of n weights."""
    return int(lib().nr_q8_quantized_size(int(n)))


def quantize_q8(weights, device: int = 0) -> bytes:
    w = np.ascontiguousarray(np.asarray(weights, dtype=np.float32).ravel())
    out = np.empty(quantized_size(w.size), np.uint8)
    check(lib().nr_quantize_q8(w.ctypes.data, w.size, out.ctypes.data, device), "nr_quantize_q8")
    return out.tobytes()


def quantize_model_file(in_path: str, out_path: str, device: int = 0) -> None:
    check(lib().nr_quantize_model_file(str(in_path).encode(), str(out_path).encode(), device),
          "nr_quantize_model_file")
