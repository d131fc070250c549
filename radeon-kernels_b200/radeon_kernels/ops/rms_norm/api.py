"""Public RMS normalisation: ``rk.rms_norm(x, weight, eps=1e-6)``.

Interface of the reference's rk.rms_norm (src/radeon_kernels/ops/rms_norm/api.py:22-61):
``x [tokens, hidden]`` and ``weight [hidden]``, CUDA fp16/bf16 on one device; operator
``"rms_norm"`` (semantic version 1.0), signature ``{dtype, tokens, hidden, eps, contiguous,
requires_grad}``, native arguments ``(x, weight, eps)``.  Winners and the fallback are this
library's kernels (``rk_rms_norm``).
"""

from __future__ import annotations

from typing import Any

from radeon_kernels.ops._common import torch_runtime
from radeon_kernels.ops._frontend import Args, dispatch
from radeon_kernels.ops._runtime import OperatorRuntime, default_operator_runtime
from radeon_kernels.providers import cuda_builtin


def _execute(x: Any, weight: Any, eps: float, *, torch_module: Any, runtime: OperatorRuntime) -> Any:
    args = Args("rms_norm", torch_module, x=x, weight=weight)
    args.tensors(x=2, weight=1).alike("x", "weight")
    tokens, hidden = args.dims("x")
    args.expect(args.dims("weight") == (hidden,), "weight must match the hidden dimension")
    eps = args.eps(eps)
    context = args.context("x", "weight")
    return dispatch(
        args, runtime, semantic_version="1.0", device_index=context.device_index,
        signature={"dtype": context.dtype, "tokens": tokens, "hidden": hidden, "eps": eps,
                   "contiguous": context.contiguous, "requires_grad": context.requires_grad},
        native_arguments=(x, weight, eps),
        fallback=cuda_builtin.rms_norm, fallback_selected=cuda_builtin.SELECTED_RMS_NORM,
    )


def rms_norm(x: Any, weight: Any, eps: float = 1e-6) -> Any:
    """Normalise each row of ``x`` by its root mean square, then scale by ``weight``."""

    return _execute(x, weight, eps, torch_module=torch_runtime("rms_norm"), runtime=default_operator_runtime())
