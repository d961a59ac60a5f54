"""Generate tests/golden/q8_tails.npz: the reference quantizer on tensors whose length is
not a multiple of 32 (and a few edge-valued full blocks), from the reference's own code.

scripts/quantize.py runs its file conversion at import time, so this script takes the
`quantize_q8` function (quantize.py:7-23) out of the file with `ast` and executes only
that definition, with the module's own imports and Q_BLOCK_SIZE.  Run where a checkout of
the reference (nvivek17/NitroRAG) is present: NITRO_REFERENCE_DIR, or a directory named
`reference` beside this repository; NumPy's
version is recorded because quantize.py's float32 arithmetic relies on NumPy's scalar
promotion rules (NumPy 2: a Python float operand keeps float32)."""
from __future__ import annotations

import ast
import os
import struct

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.environ.get("NITRO_REFERENCE_DIR") or os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(HERE))),
                                                                "reference")
REF_QUANTIZE = os.path.join(REF_DIR, "scripts", "quantize.py")
LENGTHS = [1, 5, 31, 32, 33, 64, 70, 127, 128, 129, 200, 1000]


def reference_quantize_q8():
    tree = ast.parse(open(REF_QUANTIZE).read())
    keep = [n for n in tree.body
            if isinstance(n, (ast.Import, ast.ImportFrom))
            or (isinstance(n, ast.Assign) and any(getattr(t, "id", "") == "Q_BLOCK_SIZE" for t in n.targets))
            or (isinstance(n, ast.FunctionDef) and n.name == "quantize_q8")]
    ns = {}
    exec(compile(ast.Module(body=keep, type_ignores=[]), REF_QUANTIZE, "exec"), ns)
    return ns["quantize_q8"]


def inputs():
    rng = np.random.default_rng(77)
    out = {}
    for n in LENGTHS:
        w = (rng.standard_normal(n) * 0.02).astype(np.float32)
        if n >= 33:
            w[32:min(n, 64)] = 0.0                       # an all-zero block (or tail)
        if n >= 64:
            w[:32] = np.float32(127.0) * np.linspace(-1, 1, 32, dtype=np.float32)
            w[5] = np.float32(2.5)                       # scale 1.0: exact .5 ties
            w[6] = np.float32(-3.5)
        if n >= 128:
            w[64:96] = np.float32(1e-40)                 # subnormal block
            w[100] = np.float32(3e38)                    # huge absmax
        if n % 32:
            w[-1] = np.float32(-0.75)                    # the short block's absmax, negative
        out[n] = w
    return out


def main():
    q = reference_quantize_q8()
    arrays = {"numpy_version": np.array(np.__version__)}
    for n, w in inputs().items():
        arrays[f"in_{n}"] = w
        arrays[f"out_{n}"] = np.frombuffer(bytes(q(w)), np.uint8)
    # self-check of the byte layout: scale first, then the block's bytes
    assert struct.unpack("f", bytes(arrays["out_1"][:4]))[0] == np.float32(0.75) / np.float32(127.0)
    np.savez_compressed(os.path.join(HERE, "q8_tails.npz"), **arrays)


if __name__ == "__main__":
    main()
