"""Public GEMV / skinny GEMM: ``rk.gemv(x, weight)`` computes ``x @ weight.T``.

Drop-in for src/radeon_kernels/ops/gemv/api.py:22-70: ``x`` is ``[M, K]`` with
``1 <= M <= 32``, ``weight`` is ``[N, K]`` ("nk" layout), both CUDA fp16/bf16 on one device;
the dispatch signature is ``{dtype, m, n, k, weight_layout: "nk", contiguous,
requires_grad}`` and the result is a new ``[M, N]`` tensor.  Winners and the fallback are
this library's kernels (see ``radeon_kernels.providers.cuda_builtin``).
"""

from __future__ import annotations

from typing import Any

from radeon_kernels.ops._common import tensor_context, torch_runtime, validate_same, validate_tensor
from radeon_kernels.ops._runtime import OperatorRuntime, default_operator_runtime
from radeon_kernels.providers import cuda_builtin

_SEMANTIC_VERSION = "1.0"
MAXIMUM_M = 32


def _torch() -> Any:
    return torch_runtime("gemv")


def _execute(x: Any, weight: Any, *, torch_module: Any, runtime: OperatorRuntime) -> Any:
    validate_tensor(torch_module, x, name="x", rank=2, operator="gemv")
    validate_tensor(torch_module, weight, name="weight", rank=2, operator="gemv")
    validate_same("gemv", x, weight, first_name="x", second_name="weight")
    m, k = int(x.shape[0]), int(x.shape[1])
    n, weight_k = int(weight.shape[0]), int(weight.shape[1])
    if m <= 0 or n <= 0 or k <= 0:
        raise ValueError("gemv dimensions must be positive")
    if m > MAXIMUM_M:
        raise ValueError("gemv M must be in [1, 32]")
    if weight_k != k:
        raise ValueError("gemv x and weight must share the K dimension")
    context = tensor_context(torch_module, "gemv", x, weight)
    fast = getattr(runtime, "fast_call", None)
    if fast is not None:
        # Repeated calls: the decision for this exact signature is cached (no dict,
        # no manifest scan, no pack resolution on the hot path).
        key = ("gemv", context.device_index, context.dtype, m, n, k, context.contiguous, context.requires_grad)
        result = fast(key, (x, weight))
        if result is not None:
            return result
    signature = {
        "dtype": context.dtype,
        "m": m,
        "n": n,
        "k": k,
        "weight_layout": "nk",
        "contiguous": context.contiguous,
        "requires_grad": context.requires_grad,
    }
    result = runtime.execute(
        operator="gemv",
        semantic_version=_SEMANTIC_VERSION,
        signature=signature,
        device_index=context.device_index,
        torch_module=torch_module,
        native_arguments=(x, weight),
        fallback=lambda: cuda_builtin.gemv(torch_module, x, weight),
        fallback_selected=cuda_builtin.SELECTED_GEMV,
    )
    alias = getattr(runtime, "fast_alias", None)
    if fast is not None and alias is not None:
        alias(key, runtime.fast_key("gemv", context.device_index, signature))
    return result


def gemv(x: Any, weight: Any) -> Any:
    """Compute ``x @ weight.T`` for decode GEMV and skinny GEMM (M <= 32)."""

    return _execute(x, weight, torch_module=_torch(), runtime=default_operator_runtime())
