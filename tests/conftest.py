import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

from nitrorag_b200 import synth  # noqa: E402

GOLDEN = os.path.join(ROOT, "tests", "golden")

# Tolerance of every fp32 logits comparison (the north star's bar): |a-b| <= ATOL + RTOL*|b|
RTOL = 1e-3
ATOL = 1e-4


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA engine)")
    config.addinivalue_line("markers", "slow: a long CPU-oracle comparison")


def assert_close(a, b, rtol=RTOL, atol=ATOL, what=""):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    assert a.shape == b.shape, (what, a.shape, b.shape)
    err = np.abs(a - b) - (atol + rtol * np.abs(b))
    worst = float(err.max()) if err.size else -1.0
    if worst > 0:
        i = int(np.argmax(err))
        raise AssertionError(f"{what}: mismatch at flat index {i}: got {a.ravel()[i]!r}, want {b.ravel()[i]!r} "
                             f"(max |diff| {np.abs(a - b).max():.3e})")


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    return str(tmp_path_factory.mktemp("models"))


@pytest.fixture(scope="session")
def tiny_model(model_dir):
    return synth.write_model(os.path.join(model_dir, "tiny.bin"), synth.SHAPE_TINY, seed=11)


@pytest.fixture(scope="session")
def m110_model():
    return synth.cached_model(synth.SHAPE_110M, seed=1234)


@pytest.fixture(scope="session")
def restatement():
    import oracle
    return oracle.Restatement()


def _reference(kind):
    import oracle
    if not oracle.reference_available(kind):
        pytest.skip(f"oracle/_ref/libref_{kind}.so not built (reference sources absent when building)")
    return oracle.Reference(kind)


@pytest.fixture(scope="session")
def ref_fixed():
    r = _reference("fixed")
    r.set_threads(0)
    return r


@pytest.fixture(scope="session")
def ref_faithful():
    r = _reference("faithful")
    r.set_threads(1)  # the shipped decode allocation races above one thread
    return r


def cuda_ok() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
