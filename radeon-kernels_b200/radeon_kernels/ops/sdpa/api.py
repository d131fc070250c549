"""Public scaled dot-product self-attention: ``rk.sdpa(query, key, value, *, is_causal=False,
scale=None)``.

Interface of the reference's rk.sdpa (src/radeon_kernels/ops/sdpa/api.py:22-118):
``query [batch, query_heads, sequence, head_dim]``, ``key`` / ``value`` ``[batch, kv_heads,
sequence, head_dim]`` (layout ``batch_head_sequence_dim``), equal query and key lengths,
head_dim 64, 128 or 256, query heads a multiple of the KV heads (GQA), optional causal mask,
contiguous, inference only; operator ``"sdpa"`` (semantic version 1.0) with the same
checks, messages and dispatch signature.  Where the reference falls back to torch's
``scaled_dot_product_attention`` (ops/sdpa/reference.py:39-57), the winners and the fallback
here are this library's tcgen05 kernel (``rk_sdpa``).
"""

from __future__ import annotations

from typing import Any

from radeon_kernels.ops._common import torch_runtime
from radeon_kernels.ops._frontend import Args, dispatch
from radeon_kernels.ops._runtime import OperatorRuntime, default_operator_runtime
from radeon_kernels.providers import cuda_builtin

HEAD_DIMS = (64, 128, 256)


def _execute(query: Any, key: Any, value: Any, is_causal: bool = False, scale: float | None = None, *,
             torch_module: Any, runtime: OperatorRuntime) -> Any:
    args = Args("sdpa", torch_module, query=query, key=key, value=value)
    args.tensors(query=4, key=4, value=4).alike("query", "key", "value")
    args.expect(isinstance(is_causal, bool), "is_causal must be bool", TypeError)
    batch, query_heads, sequence, head_dim = args.dims("query")
    kv_batch, kv_heads, kv_sequence, kv_head_dim = args.dims("key")
    args.expect(args.dims("value") == args.dims("key"), "key and value must have the same shape")
    args.expect(min(batch, query_heads, sequence, kv_heads) > 0, "tensor dimensions must be positive")
    args.expect(kv_batch == batch, "query, key and value must share the batch dimension")
    args.expect(kv_sequence == sequence, "1.0 requires equal query and KV sequence lengths")
    args.expect(kv_head_dim == head_dim and head_dim in HEAD_DIMS, "head_dim must match and be one of 64, 128, 256")
    args.expect(query_heads % kv_heads == 0, "query_heads must be divisible by kv_heads")
    context = args.inference_only("query", "key", "value")
    scale, scale_mode = args.scale(scale, head_dim)
    signature = {
        "dtype": context.dtype, "batch": batch, "query_heads": query_heads, "kv_heads": kv_heads,
        "sequence": sequence, "head_dim": head_dim, "layout": "batch_head_sequence_dim",
        "attention_mode": "causal" if is_causal else "noncausal", "scale_mode": scale_mode,
        "contiguous": True, "requires_grad": False,
    }
    return dispatch(
        args, runtime, semantic_version="1.0", signature=signature, device_index=context.device_index,
        native_arguments=(query, key, value, is_causal, scale),
        fallback=cuda_builtin.sdpa, fallback_selected=cuda_builtin.SELECTED_SDPA,
    )


def sdpa(query: Any, key: Any, value: Any, *, is_causal: bool = False, scale: float | None = None) -> Any:
    """Run inference-only scaled dot-product self-attention with optional GQA."""

    return _execute(query, key, value, is_causal, scale, torch_module=torch_runtime("sdpa"),
                    runtime=default_operator_runtime())
