"""The GPU Q8_0 quantizer (quantize.cu) through the C ABI, byte for byte against the
reference's scripts/quantize.py (golden files made by running it) and against the CPU
restatement (oracle/nitro_oracle.cpp, pinned to the same goldens) at larger sizes."""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from nitrorag_b200 import NrError, quantize_model_file, quantize_q8, quantized_size, synth
from nitrorag_b200._lib import lib

pytestmark = pytest.mark.gpu


def _crafted(n, seed):
    """N(0, 0.02) weights with edge blocks sprinkled in: all zero, exact .5 ties at scale 1,
    subnormal, huge, a negative absmax."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal(n) * 0.02).astype(np.float32)
    nb = n // 32
    for kind, blocks in enumerate(np.array_split(rng.choice(nb, size=min(nb, 400), replace=False), 5)):
        for b in blocks:
            blk = w[32 * b:32 * b + 32]
            if kind == 0:
                blk[:] = 0.0
            elif kind == 1:
                blk[:] = np.float32(127.0) * np.linspace(-1, 1, 32, dtype=np.float32)
                blk[3] = np.float32(0.5)
                blk[4] = np.float32(-2.5)
            elif kind == 2:
                blk[:] = np.float32(3e-41) * rng.standard_normal(32).astype(np.float32)
            elif kind == 3:
                blk[7] = np.float32(-2e38)
            else:
                blk[:] = -np.abs(blk)
    return w


def test_model_file_matches_reference_script(tmp_path):
    """nr_quantize_model_file on the golden fp32 checkpoint reproduces the Q8_0 file that
    scripts/quantize.py wrote from it."""
    meta = json.load(open(os.path.join(GOLDEN, "golden.json")))["quantizer"]
    want = open(os.path.join(GOLDEN, meta["output"]), "rb").read()
    out = tmp_path / "q8.bin"
    quantize_model_file(os.path.join(GOLDEN, meta["input"]), str(out))
    got = out.read_bytes()
    assert hashlib.sha256(got).hexdigest() == meta["output_sha256"]
    assert got == want


def test_short_last_blocks_match_reference():
    g = np.load(os.path.join(GOLDEN, "q8_tails.npz"))
    for k in g.files:
        if k.startswith("in_"):
            n = int(k[3:])
            assert quantize_q8(g[k]) == g[f"out_{n}"].tobytes(), n


@pytest.mark.parametrize("n", [128, 4096 + 64, 12_582_912 + 77])
def test_device_entry_matches_restatement(restatement, n):
    """Device buffers: full groups of 128 weights on the vector path, the tail (whole and
    short blocks) on the scalar path."""
    w = _crafted(n, seed=n)
    want = restatement.quantize_q8(w)
    dw = torch.from_numpy(w).cuda()
    out = torch.zeros(quantized_size(n), dtype=torch.uint8, device="cuda")
    rc = lib().nr_quantize_q8_device(dw.data_ptr(), n, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    got = out.cpu().numpy().tobytes()
    if got != want:
        diff = np.flatnonzero(np.frombuffer(got, np.uint8) != np.frombuffer(want, np.uint8))
        raise AssertionError(f"{diff.size} bytes differ, first at {diff[0]} (block {diff[0] // 36})")


def test_host_entry_spans_pipeline_pieces(restatement):
    """Host buffers larger than one pinned slot (32 M weights): three pieces, the last one
    ending in a short block."""
    n = 70 * (1 << 20) + 45
    w = _crafted(n, seed=3)
    assert quantize_q8(w) == restatement.quantize_q8(w)


def test_fp32_checkpoint_converts_to_the_generated_model(tmp_path):
    """A seeded fp32 checkpoint quantized on the GPU equals the Q8_0 model the generator
    writes for the same seed (its tensors go through the vectorised host restatement)."""
    q8 = synth.write_model(str(tmp_path / "m.bin"), synth.SHAPE_TINY, seed=9, fp32_path=str(tmp_path / "m32.bin"))
    quantize_model_file(str(tmp_path / "m32.bin"), str(tmp_path / "gpu.bin"))
    assert (tmp_path / "gpu.bin").read_bytes() == open(q8, "rb").read()


def test_argument_errors(tmp_path):
    dw = torch.zeros(64, dtype=torch.float32, device="cuda")
    out = torch.zeros(72, dtype=torch.uint8, device="cuda")
    # misaligned input pointer: refused before any launch
    assert lib().nr_quantize_q8_device(dw.data_ptr() + 4, 32, out.data_ptr(), None) == -1
    with pytest.raises(NrError, match="NR_ERR_IO"):
        quantize_model_file(str(tmp_path / "missing.bin"), str(tmp_path / "o.bin"))
    bad = tmp_path / "bad.bin"
    bad.write_bytes(np.array([64, 64, 1, 0, 1, 16, 4], np.int32).tobytes())  # n_heads 0
    with pytest.raises(NrError, match="NR_ERR_FORMAT"):
        quantize_model_file(str(bad), str(tmp_path / "o.bin"))
    short = tmp_path / "short.bin"
    short.write_bytes(np.array([64, 64, 1, 1, 1, 16, 4], np.int32).tobytes() + b"\0" * 100)
    with pytest.raises(NrError, match="NR_ERR_FORMAT"):
        quantize_model_file(str(short), str(tmp_path / "o.bin"))
