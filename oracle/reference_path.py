"""The reference's own CPU path for rk.gemm / rk.gemv, restated -- TEST INFRASTRUCTURE ONLY.

These are the functions the reference executes when no native winner matches, i.e. the
path the reference runs on CPU tensors (``rk.gemm`` itself rejects CPU tensors at
ops/gemm/api.py:62-63, so the baseline calls them directly):

* ``gemm_fallback``  -- providers/torch_fallback.py:6-9
* ``gemv_fallback``  -- ops/gemv/reference.py:12-15
* ``gemv_reference`` -- ops/gemv/reference.py:6-9 (the gemv contract's declared oracle)
* ``silu_mul_reference`` -- ops/swiglu/reference.py:6-9
* ``rms_norm_reference`` -- ops/rms_norm/reference.py:6-10
* ``add_rms_norm_reference`` -- ops/add_rms_norm/reference.py:8-12
* ``paged_attention_decode_reference`` -- ops/paged_attention/reference.py:8-47
* ``gemm_swiglu_reference`` -- no single reference function: the fused FFN-up operator's
  definition, the reference's GEMM and silu_mul composed in fp32

They are one-line calls of ``torch.mm``; torch is the reference's arithmetic engine (see
``rk_oracle.c`` for the version note).  ``bench.py --impl reference`` times them on the
host cores as the reference arm; tests compare the CUDA path against them.
"""

from __future__ import annotations

from typing import Any


def gemm_fallback(torch_module: Any, a: Any, b: Any, output: Any | None = None) -> Any:
    return torch_module.mm(a, b) if output is None else torch_module.mm(a, b, out=output)


def gemv_fallback(torch_module: Any, x: Any, weight: Any) -> Any:
    return torch_module.mm(x, weight.transpose(0, 1))


def gemv_reference(torch_module: Any, x: Any, weight: Any) -> Any:
    return torch_module.mm(x.float(), weight.float().transpose(0, 1)).to(dtype=x.dtype)


def gemm_reference_fp32(torch_module: Any, a: Any, b: Any) -> Any:
    """fp32-accumulated product before the final rounding (parity metric denominator)."""

    return torch_module.mm(a.float(), b.float())


def silu_mul_reference(torch_module: Any, gate: Any, up: Any) -> Any:
    g = gate.float()
    return (g * torch_module.sigmoid(g) * up.float()).to(dtype=gate.dtype)


def rms_norm_reference(torch_module: Any, x: Any, weight: Any, eps: float) -> Any:
    v = x.float()
    scale = torch_module.rsqrt(v.square().mean(dim=-1, keepdim=True) + eps)
    return (v * scale * weight.float()).to(dtype=x.dtype)


def add_rms_norm_reference(torch_module: Any, x: Any, residual: Any, weight: Any, eps: float) -> tuple[Any, Any]:
    residual_out = x + residual
    return rms_norm_reference(torch_module, residual_out, weight, eps), residual_out


def gemm_swiglu_reference(torch_module: Any, a: Any, b: Any) -> Any:
    n = int(b.shape[1]) // 2
    y = torch_module.mm(a.float(), b.float())
    g, u = y[:, :n], y[:, n:]
    return (g * torch_module.sigmoid(g) * u).to(dtype=a.dtype)


def paged_attention_decode_reference(
    torch_module: Any, query: Any, key_cache: Any, value_cache: Any, block_tables: Any, context_lengths: Any, scale: float
) -> Any:
    batch, heads, head_dim = (int(n) for n in query.shape)
    block_size, kv_heads = int(key_cache.shape[1]), int(key_cache.shape[2])
    max_ctx = int(block_tables.shape[1]) * block_size
    positions = torch_module.arange(max_ctx, device=query.device)
    slots = block_tables.long().index_select(1, positions // block_size) * block_size + (positions % block_size).unsqueeze(0)
    keys = key_cache.view(-1, kv_heads, head_dim).index_select(0, slots.reshape(-1)).view(batch, max_ctx, kv_heads, head_dim)
    values = value_cache.view(-1, kv_heads, head_dim).index_select(0, slots.reshape(-1)).view(batch, max_ctx, kv_heads, head_dim)
    kv_index = torch_module.arange(heads, device=query.device) // (heads // kv_heads)
    keys = keys.index_select(2, kv_index).float()
    values = values.index_select(2, kv_index).float()
    scores = torch_module.einsum("bhd,bthd->bht", query.float(), keys) * scale
    valid = positions.unsqueeze(0) < context_lengths.long().unsqueeze(1)
    scores = scores.masked_fill(~valid.unsqueeze(1), float("-inf"))
    probabilities = torch_module.softmax(scores, dim=-1, dtype=torch_module.float32)
    return torch_module.einsum("bht,bthd->bhd", probabilities, values).to(dtype=query.dtype)


def sdpa_reference(torch_module: Any, query: Any, key: Any, value: Any, is_causal: bool, scale: float) -> Any:
    """The reference's fp32 self-attention definition (ops/sdpa/reference.py:13-36): K and V
    repeated to the query heads, fp32 scores times scale, causal mask from tril, fp32
    softmax, probabilities times V, cast to the query dtype."""

    group = int(query.shape[1]) // int(key.shape[1])
    keys = key.repeat_interleave(group, dim=1).float() if group > 1 else key.float()
    values = value.repeat_interleave(group, dim=1).float() if group > 1 else value.float()
    scores = torch_module.matmul(query.float(), keys.transpose(-2, -1)) * scale
    if is_causal:
        seq = int(query.shape[2])
        keep = torch_module.ones((seq, seq), device=query.device, dtype=torch_module.bool).tril()
        scores = scores.masked_fill(~keep, float("-inf"))
    probabilities = torch_module.softmax(scores, dim=-1, dtype=torch_module.float32)
    return torch_module.matmul(probabilities, values).to(dtype=query.dtype)

