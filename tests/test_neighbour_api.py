"""rk.silu_mul / rk.rms_norm / rk.add_rms_norm front-ends on CPU: signatures, validation
order and messages (the reference's tests/test_llm_ops.py checks the same contract with a
fake torch)."""

from __future__ import annotations

import pytest

from fakes import FakeTensor, FakeTorch
from radeon_kernels.ops.add_rms_norm.api import _execute as execute_add_rms_norm
from radeon_kernels.ops.rms_norm.api import _execute as execute_rms_norm
from radeon_kernels.ops.swiglu.api import _execute as execute_silu_mul


class CaptureRuntime:
    def __init__(self, result="result"):
        self.call = None
        self.result = result

    def execute(self, **kwargs):
        self.call = kwargs
        return self.result


def test_rms_norm_signature():
    runtime = CaptureRuntime()
    x = FakeTensor((128, 4096), requires_grad=True)
    assert execute_rms_norm(x, FakeTensor((4096,)), 1e-6, torch_module=FakeTorch(), runtime=runtime) == "result"
    assert runtime.call["operator"] == "rms_norm"
    assert runtime.call["semantic_version"] == "1.0"
    assert runtime.call["signature"] == {
        "dtype": "fp16",
        "tokens": 128,
        "hidden": 4096,
        "eps": 1e-6,
        "contiguous": True,
        "requires_grad": True,
    }
    assert runtime.call["fallback_selected"] == "cuda/rms_norm"
    assert runtime.call["native_arguments"][-1] == 1e-6


def test_add_rms_norm_returns_two_outputs_and_passes_eps_last():
    runtime = CaptureRuntime(["normalized", "residual"])
    tensors = (FakeTensor((32, 8192)), FakeTensor((32, 8192)), FakeTensor((8192,)))
    result = execute_add_rms_norm(*tensors, 1e-6, torch_module=FakeTorch(), runtime=runtime)
    assert result == ("normalized", "residual")
    assert runtime.call["operator"] == "add_rms_norm"
    assert runtime.call["native_arguments"][-1] == 1e-6
    assert runtime.call["fallback_selected"] == "cuda/add_rms_norm"


def test_add_rms_norm_rejects_a_single_output():
    runtime = CaptureRuntime("only-one")
    tensors = (FakeTensor((2, 8)), FakeTensor((2, 8)), FakeTensor((8,)))
    with pytest.raises(RuntimeError, match="must return two tensors"):
        execute_add_rms_norm(*tensors, 1e-6, torch_module=FakeTorch(), runtime=runtime)


def test_silu_mul_maps_to_the_versioned_swiglu_operator():
    runtime = CaptureRuntime()
    execute_silu_mul(FakeTensor((1, 11008)), FakeTensor((1, 11008)), torch_module=FakeTorch(), runtime=runtime)
    assert runtime.call["operator"] == "swiglu"
    assert runtime.call["signature"] == {
        "dtype": "fp16",
        "tokens": 1,
        "hidden": 11008,
        "contiguous": True,
        "requires_grad": False,
    }
    assert runtime.call["fallback_selected"] == "cuda/silu_mul"


@pytest.mark.parametrize(
    "call, exc, message",
    [
        (lambda t, r: execute_rms_norm(FakeTensor((2, 8)), FakeTensor((4,)), 1e-6, torch_module=t, runtime=r), ValueError, "hidden dimension"),
        (lambda t, r: execute_rms_norm(FakeTensor((2, 8)), FakeTensor((8,)), 0, torch_module=t, runtime=r), ValueError, "positive and finite"),
        (lambda t, r: execute_rms_norm(FakeTensor((2, 8)), FakeTensor((8,)), float("nan"), torch_module=t, runtime=r), ValueError, "positive and finite"),
        (lambda t, r: execute_rms_norm(FakeTensor((2, 8)), FakeTensor((8,)), True, torch_module=t, runtime=r), TypeError, "eps must be a number"),
        (lambda t, r: execute_rms_norm(FakeTensor((8,)), FakeTensor((8,)), 1e-6, torch_module=t, runtime=r), ValueError, "x must be rank 2"),
        (lambda t, r: execute_add_rms_norm(FakeTensor((2, 8)), FakeTensor((3, 8)), FakeTensor((8,)), 1e-6, torch_module=t, runtime=r), ValueError, "same shape"),
        (lambda t, r: execute_add_rms_norm(FakeTensor((2, 8)), FakeTensor((2, 8), dtype="bfloat16"), FakeTensor((8,)), 1e-6, torch_module=t, runtime=r), TypeError, "same dtype"),
        (lambda t, r: execute_silu_mul(FakeTensor((2, 8)), FakeTensor((2, 9)), torch_module=t, runtime=r), ValueError, "same shape"),
        (lambda t, r: execute_silu_mul(FakeTensor((2, 8), dtype="float32"), FakeTensor((2, 8), dtype="float32"), torch_module=t, runtime=r), TypeError, "float16 and torch.bfloat16"),
    ],
)
def test_invalid_calls_raise_before_dispatch(call, exc, message):
    runtime = CaptureRuntime()
    with pytest.raises(exc, match=message):
        call(FakeTorch(), runtime)
    assert runtime.call is None
