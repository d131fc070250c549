"""Public fused residual add + RMS normalisation: ``rk.add_rms_norm(x, residual, weight, eps)``.

Interface of the reference's rk.add_rms_norm (src/radeon_kernels/ops/add_rms_norm/api.py:
22-79): ``x`` and ``residual`` ``[tokens, hidden]``, ``weight [hidden]``, CUDA fp16/bf16 on
one device; operator ``"add_rms_norm"`` (semantic version 1.0), signature ``{dtype, tokens,
hidden, eps, contiguous, requires_grad}``.  Returns ``(normalized, residual_out)`` with
``residual_out = x + residual`` (rounded to the dtype) and ``normalized =
rms_norm(residual_out, weight, eps)``.  Winners and the fallback are this library's kernels
(``rk_add_rms_norm``).
"""

from __future__ import annotations

from typing import Any

from radeon_kernels.ops._common import torch_runtime
from radeon_kernels.ops._frontend import Args, dispatch
from radeon_kernels.ops._runtime import OperatorRuntime, default_operator_runtime
from radeon_kernels.providers import cuda_builtin


def _execute(x: Any, residual: Any, weight: Any, eps: float, *, torch_module: Any,
             runtime: OperatorRuntime) -> tuple[Any, Any]:
    args = Args("add_rms_norm", torch_module, x=x, residual=residual, weight=weight)
    args.tensors(x=2, residual=2, weight=1)
    args.alike("x", "residual")
    args.alike("x", "weight")
    tokens, hidden = args.dims("x")
    args.expect(args.dims("residual") == (tokens, hidden), "x and residual must have the same shape")
    args.expect(args.dims("weight") == (hidden,), "weight must match the hidden dimension")
    eps = args.eps(eps)
    context = args.context("x", "residual", "weight")
    outputs = dispatch(
        args, runtime, semantic_version="1.0", device_index=context.device_index,
        signature={"dtype": context.dtype, "tokens": tokens, "hidden": hidden, "eps": eps,
                   "contiguous": context.contiguous, "requires_grad": context.requires_grad},
        native_arguments=(x, residual, weight, eps),
        fallback=cuda_builtin.add_rms_norm, fallback_selected=cuda_builtin.SELECTED_ADD_RMS_NORM,
    )
    if not isinstance(outputs, (tuple, list)) or len(outputs) != 2:
        raise RuntimeError("add_rms_norm implementation must return two tensors")
    normalized, residual_out = outputs
    return normalized, residual_out


def add_rms_norm(x: Any, residual: Any, weight: Any, eps: float = 1e-6) -> tuple[Any, Any]:
    """Add a residual and RMS-normalise it, returning ``(normalized, residual_out)``."""

    return _execute(x, residual, weight, eps, torch_module=torch_runtime("add_rms_norm"),
                    runtime=default_operator_runtime())
