"""The GPU quantizer's entry points on a machine without a GPU: they fail loudly (no CPU
path) and validate their arguments before touching the device."""
import pytest

from nitrorag_b200 import NrError, quantize_model_file, quantize_q8, quantized_size


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


def test_quantized_size():
    assert [quantized_size(n) for n in (0, 1, 31, 32, 33, 64, 70)] == [0, 5, 35, 36, 41, 72, 82]


@pytest.mark.skipif(_has_gpu(), reason="checks the no-GPU error path")
def test_no_device_is_an_error(tmp_path):
    with pytest.raises(NrError, match="NR_ERR_NO_DEVICE"):
        quantize_q8([0.5] * 64)
    src = tmp_path / "in.bin"
    src.write_bytes(b"\0" * 64)
    with pytest.raises(NrError, match="NR_ERR_NO_DEVICE"):
        quantize_model_file(str(src), str(tmp_path / "out.bin"))
