"""rk.gemv front-end on CPU: signature, validation order and messages."""

from __future__ import annotations

import pytest

from fakes import FakeTensor, FakeTorch
from radeon_kernels.ops.gemv.api import _execute


class CaptureRuntime:
    def __init__(self):
        self.call = None

    def execute(self, **kwargs):
        self.call = kwargs
        return "result"


def test_signature_uses_nk_layout():
    runtime = CaptureRuntime()
    assert _execute(FakeTensor((8, 4096)), FakeTensor((11008, 4096)), torch_module=FakeTorch(), runtime=runtime) == "result"
    assert runtime.call["operator"] == "gemv"
    assert runtime.call["signature"] == {
        "dtype": "fp16",
        "m": 8,
        "n": 11008,
        "k": 4096,
        "weight_layout": "nk",
        "contiguous": True,
        "requires_grad": False,
    }
    assert runtime.call["fallback_selected"] == "cuda/gemv"
    assert runtime.call["native_arguments"][0].shape == (8, 4096)


def test_signature_records_layout_flags():
    runtime = CaptureRuntime()
    _execute(
        FakeTensor((1, 64), dtype="bfloat16", contiguous=False),
        FakeTensor((32, 64), dtype="bfloat16", requires_grad=True),
        torch_module=FakeTorch(),
        runtime=runtime,
    )
    sig = runtime.call["signature"]
    assert (sig["dtype"], sig["contiguous"], sig["requires_grad"]) == ("bf16", False, True)


@pytest.mark.parametrize(
    "x, w, exc, message",
    [
        ((1, 4096), (4096, 8192), ValueError, "share the K dimension"),
        ((33, 4096), (4096, 4096), ValueError, "M must be in"),
        ((0, 4096), (4096, 4096), ValueError, "dimensions must be positive"),
        ((4096,), (4096, 4096), ValueError, "x must be rank 2"),
    ],
)
def test_invalid_calls(x, w, exc, message):
    with pytest.raises(exc, match=message):
        _execute(FakeTensor(x), FakeTensor(w), torch_module=FakeTorch(), runtime=CaptureRuntime())


def test_dtype_and_device_mismatch():
    with pytest.raises(TypeError, match="same dtype"):
        _execute(FakeTensor((1, 8)), FakeTensor((8, 8), dtype="bfloat16"), torch_module=FakeTorch(), runtime=CaptureRuntime())
    cpu = FakeTensor((1, 8))
    cpu.is_cuda = False
    with pytest.raises(ValueError, match="visible CUDA GPU"):
        _execute(cpu, FakeTensor((8, 8)), torch_module=FakeTorch(), runtime=CaptureRuntime())
