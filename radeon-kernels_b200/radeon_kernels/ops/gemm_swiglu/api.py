"""Fused FFN-up projection with SwiGLU: ``rk.gemm_swiglu(a, w_gate_up)``.

Computes ``silu(a @ w_gate_up[:, :N]) * (a @ w_gate_up[:, N:])`` for ``a [M, K]`` and
``w_gate_up [K, 2N]`` (the gate and up projections side by side, ``torch.cat([w_gate,
w_up], dim=1)``), CUDA fp16/bf16 on one device; the result is a new ``[M, N]`` tensor.

No counterpart in the reference, where an FFN runs ``rk.gemm`` into ``[M, 2N]`` and then
``rk.silu_mul`` (src/radeon_kernels/ops/gemm/api.py, ops/swiglu/api.py).  Here both products
accumulate in fp32 in tensor memory and the GEMM epilogue applies ``silu(g) * u`` to the fp32
sums before the single rounding, so the ``[M, 2N]`` intermediate never reaches HBM.  It runs
through the same dispatch runtime (operator ``"gemm_swiglu"``, semantic version 1.0,
signature ``{dtype, layout: "nn", m, n, k, contiguous, requires_grad}``); shapes the fused
kernel cannot take (N or K not a multiple of 8, unaligned views) run this library's GEMM and
``silu_mul`` kernels one after the other.
"""

from __future__ import annotations

from typing import Any

from radeon_kernels.ops._common import tensor_context, torch_runtime, validate_same, validate_tensor
from radeon_kernels.ops._runtime import OperatorRuntime, default_operator_runtime
from radeon_kernels.providers import cuda_builtin

_SEMANTIC_VERSION = "1.0"


def _torch() -> Any:
    return torch_runtime("gemm_swiglu")


def _execute(a: Any, b: Any, *, torch_module: Any, runtime: OperatorRuntime) -> Any:
    validate_tensor(torch_module, a, name="a", rank=2, operator="gemm_swiglu")
    validate_tensor(torch_module, b, name="b", rank=2, operator="gemm_swiglu")
    validate_same("gemm_swiglu", a, b, first_name="a", second_name="b")
    m, k = int(a.shape[0]), int(a.shape[1])
    k2, n2 = int(b.shape[0]), int(b.shape[1])
    if k != k2:
        raise ValueError("gemm_swiglu a and b must share the K dimension")
    if n2 % 2 != 0 or n2 == 0:
        raise ValueError("gemm_swiglu b must hold the gate and up projections side by side (2N columns)")
    context = tensor_context(torch_module, "gemm_swiglu", a, b)
    signature = {
        "dtype": context.dtype,
        "layout": "nn",
        "m": m,
        "n": n2 // 2,
        "k": k,
        "contiguous": context.contiguous,
        "requires_grad": context.requires_grad,
    }
    return runtime.execute(
        operator="gemm_swiglu",
        semantic_version=_SEMANTIC_VERSION,
        signature=signature,
        device_index=context.device_index,
        torch_module=torch_module,
        native_arguments=(a, b),
        fallback=lambda: cuda_builtin.gemm_swiglu(torch_module, a, b),
        fallback_selected=cuda_builtin.SELECTED_GEMM_SWIGLU,
    )


def gemm_swiglu(a: Any, w_gate_up: Any) -> Any:
    """``silu(a @ w_gate_up[:, :N]) * (a @ w_gate_up[:, N:])`` in one kernel."""

    return _execute(a, w_gate_up, torch_module=_torch(), runtime=default_operator_runtime())
