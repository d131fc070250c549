"""Public paged decode attention: ``rk.paged_attention_decode(query, key_cache, value_cache,
block_tables, context_lengths, scale=None)``.

Interface of the reference's rk.paged_attention_decode (src/radeon_kernels/ops/paged_attention/api.py:38-157): ``query [batch, query_heads,
head_dim]``; ``key_cache`` / ``value_cache`` ``[num_blocks, block_size, kv_heads, head_dim]``
(layout ``block_slot_head_dim``); ``block_tables [batch, max_blocks]`` and ``context_lengths
[batch]`` int32/int64; head_dim 64, 128 or 256; query heads a multiple of the KV heads;
contiguous, inference only.  Operator ``"paged_attention_decode"`` (semantic version 1.0) with
the reference's signature.  Winners and the fallback are this library's kernel
(``rk_paged_attention_decode``).
"""

from __future__ import annotations

from typing import Any

from radeon_kernels.ops._common import torch_runtime
from radeon_kernels.ops._frontend import Args, dispatch
from radeon_kernels.ops._runtime import OperatorRuntime, default_operator_runtime
from radeon_kernels.providers import cuda_builtin

HEAD_DIMS = (64, 128, 256)


def _execute(query: Any, key_cache: Any, value_cache: Any, block_tables: Any, context_lengths: Any,
             scale: float | None = None, *, torch_module: Any, runtime: OperatorRuntime) -> Any:
    args = Args("paged_attention_decode", torch_module, query=query, key_cache=key_cache,
                value_cache=value_cache, block_tables=block_tables, context_lengths=context_lengths)
    args.tensors(query=3, key_cache=4, value_cache=4).alike("query", "key_cache", "value_cache")
    args.expect(args.dims("key_cache") == args.dims("value_cache"), "key_cache and value_cache must have the same shape")
    args.indices(block_tables=2, context_lengths=1)
    args.expect(block_tables.device == query.device and context_lengths.device == query.device,
                "index tensors must use the same device as query")
    args.expect(block_tables.dtype == context_lengths.dtype, "block_tables and context_lengths must use the same dtype",
                TypeError)
    batch, query_heads, head_dim = args.dims("query")
    num_blocks, block_size, kv_heads, cache_head_dim = args.dims("key_cache")
    table_rows, max_blocks = args.dims("block_tables")
    args.expect(min(batch, query_heads, num_blocks, block_size, kv_heads) > 0, "tensor dimensions must be positive")
    args.expect(cache_head_dim == head_dim and head_dim in HEAD_DIMS,
                "head_dim must match cache and be one of 64, 128, 256")
    args.expect(query_heads % kv_heads == 0, "query_heads must be divisible by kv_heads")
    args.expect(table_rows == batch and max_blocks > 0, "block_tables must have shape [batch, max_blocks]")
    args.expect(args.dims("context_lengths") == (batch,), "context_lengths must contain one length per sequence")
    context = args.inference_only("query", "key_cache", "value_cache", "block_tables", "context_lengths")
    scale, scale_mode = args.scale(scale, head_dim)
    signature = {
        "dtype": context.dtype, "batch": batch, "query_heads": query_heads, "kv_heads": kv_heads,
        "head_dim": head_dim, "num_blocks": num_blocks, "block_size": block_size,
        "max_blocks_per_sequence": max_blocks, "index_dtype": args.index_dtype("block_tables"),
        "cache_layout": "block_slot_head_dim", "scale_mode": scale_mode, "contiguous": True,
        "requires_grad": False,
    }
    return dispatch(
        args, runtime, semantic_version="1.0", signature=signature, device_index=context.device_index,
        native_arguments=(query, key_cache, value_cache, block_tables, context_lengths, scale),
        fallback=cuda_builtin.paged_attention_decode, fallback_selected=cuda_builtin.SELECTED_PAGED_ATTENTION,
    )


def paged_attention_decode(query: Any, key_cache: Any, value_cache: Any, block_tables: Any,
                           context_lengths: Any, scale: float | None = None) -> Any:
    """Attend one query token per sequence over a paged K/V cache."""

    return _execute(query, key_cache, value_cache, block_tables, context_lengths, scale,
                    torch_module=torch_runtime("paged_attention_decode"), runtime=default_operator_runtime())
