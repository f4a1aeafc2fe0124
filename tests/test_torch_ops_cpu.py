"""The PyTorch custom operators (quickruncuda_b200/torch_ops.py) without a
GPU: they register under torch.ops.qrc, their fake implementations give the
shapes and dtypes torch.compile traces with, and a CPU tensor is refused
rather than computed some other way."""
import pytest
import torch

import quickruncuda_b200.torch_ops  # noqa: F401  (registers torch.ops.qrc.*)
from torch._subclasses.fake_tensor import FakeTensorMode


def test_registered():
    assert hasattr(torch.ops.qrc, "absmax")
    assert hasattr(torch.ops.qrc, "amax_quant_e4m3")
    assert hasattr(torch.ops.qrc, "reduce")


@pytest.mark.parametrize("shape", [(0,), (7,), (3, 5), (2, 3, 4)])
def test_fake_shapes(shape):
    with FakeTensorMode():
        x = torch.empty(shape, device="cuda")
        y = torch.ops.qrc.absmax(x)
        assert y.shape == () and y.dtype == torch.float32 and y.device.type == "cuda"
        assert torch.ops.qrc.reduce(x, "sum").dtype == torch.float64
        assert torch.ops.qrc.reduce(x, "min").dtype == torch.float32
        xb = torch.empty(shape, device="cuda", dtype=torch.bfloat16)
        q, scale, amax = torch.ops.qrc.amax_quant_e4m3(xb)
        assert q.shape == xb.shape and q.dtype == torch.float8_e4m3fn
        assert scale.shape == () and amax.shape == () and scale.dtype == torch.float32


def test_cpu_tensor_is_refused():
    with pytest.raises(NotImplementedError):
        torch.ops.qrc.absmax(torch.ones(3))
    with pytest.raises(NotImplementedError):
        torch.ops.qrc.amax_quant_e4m3(torch.ones(3, dtype=torch.bfloat16))
