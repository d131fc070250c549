"""rk.sdpa front-end on CPU: signature, validation order and messages of the reference's
operator (src/radeon_kernels/ops/sdpa/api.py:22-118), checked with a fake torch."""

from __future__ import annotations

import math

import pytest

from fakes import FakeTensor, FakeTorch
from radeon_kernels.ops.sdpa.api import _execute as execute_sdpa


class CaptureRuntime:
    def __init__(self):
        self.call = None

    def execute(self, **kwargs):
        self.call = kwargs
        return "result"


def _qkv(b=1, hq=32, hkv=8, s=512, d=128, **kw):
    return FakeTensor((b, hq, s, d), **kw), FakeTensor((b, hkv, s, d)), FakeTensor((b, hkv, s, d))


def test_signature_and_native_arguments():
    runtime = CaptureRuntime()
    q, k, v = _qkv()
    assert execute_sdpa(q, k, v, True, None, torch_module=FakeTorch(), runtime=runtime) == "result"
    call = runtime.call
    assert call["operator"] == "sdpa" and call["semantic_version"] == "1.0"
    assert call["signature"] == {
        "dtype": "fp16",
        "batch": 1,
        "query_heads": 32,
        "kv_heads": 8,
        "sequence": 512,
        "head_dim": 128,
        "layout": "batch_head_sequence_dim",
        "attention_mode": "causal",
        "scale_mode": "default",
        "contiguous": True,
        "requires_grad": False,
    }
    assert call["native_arguments"][3] is True
    assert call["native_arguments"][4] == pytest.approx(1 / math.sqrt(128))
    assert call["fallback_selected"] == "cuda/sdpa"
    execute_sdpa(q, k, v, False, 0.25, torch_module=FakeTorch(), runtime=runtime)
    assert runtime.call["signature"]["attention_mode"] == "noncausal"
    assert runtime.call["signature"]["scale_mode"] == "explicit"
    assert runtime.call["native_arguments"][4] == 0.25


@pytest.mark.parametrize(
    "args, exc, message",
    [
        ((FakeTensor((1, 2, 8)), FakeTensor((1, 2, 8, 64)), FakeTensor((1, 2, 8, 64)), False, None), ValueError, "query must be rank 4"),
        (_qkv() + ("yes", None), TypeError, "is_causal must be bool"),
        ((FakeTensor((1, 2, 8, 64)), FakeTensor((1, 2, 8, 64)), FakeTensor((1, 2, 9, 64)), False, None), ValueError, "same shape"),
        ((FakeTensor((1, 2, 8, 64)), FakeTensor((2, 2, 8, 64)), FakeTensor((2, 2, 8, 64)), False, None), ValueError, "batch dimension"),
        ((FakeTensor((1, 2, 8, 64)), FakeTensor((1, 2, 9, 64)), FakeTensor((1, 2, 9, 64)), False, None), ValueError, "equal query and KV sequence"),
        ((FakeTensor((1, 2, 8, 96)), FakeTensor((1, 2, 8, 96)), FakeTensor((1, 2, 8, 96)), False, None), ValueError, "one of 64, 128, 256"),
        ((FakeTensor((1, 3, 8, 64)), FakeTensor((1, 2, 8, 64)), FakeTensor((1, 2, 8, 64)), False, None), ValueError, "divisible by kv_heads"),
        (_qkv(requires_grad=True) + (False, None), ValueError, "inference-only"),
        (_qkv() + (False, 0.0), ValueError, "positive and finite"),
        (_qkv() + (False, True), TypeError, "scale must be a number"),
    ],
)
def test_invalid_calls_raise_before_dispatch(args, exc, message):
    runtime = CaptureRuntime()
    with pytest.raises(exc, match=message):
        execute_sdpa(*args, torch_module=FakeTorch(), runtime=runtime)
    assert runtime.call is None
