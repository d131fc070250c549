"""The built-in ``cuda`` provider: the always-available fallback of every manifest.

Where the reference falls back to ``torch.mm`` (src/radeon_kernels/providers/torch_fallback.py:6-9,
src/radeon_kernels/ops/gemv/reference.py:12-15), this build falls back to its own CUDA
kernels through the compiled binding, with the ``auto`` variant: the tcgen05 GEMM or the
streaming GEMV when shape and alignment allow, the generic predicated kernels otherwise.
So every call on a GPU, matched by a dispatch entry or not, runs a kernel of this
library; nothing falls back to a vendor library or to the CPU.

GEMM operands that are transposed views of dense matrices (``x.t()``) are read in place
through ``rk_gemm_layout`` (the "nt"/"tn" layouts); other non-contiguous inputs are packed
first (a device copy).  Inputs that require gradients go through :class:`_GemmFunction` /
:class:`_GemvFunction`, whose backward GEMMs read the saved operands transposed in place.
"""

from __future__ import annotations

from typing import Any

from radeon_kernels import _native

SELECTED_GEMM = "cuda/gemm"
SELECTED_GEMV = "cuda/gemv"
SELECTED_SILU_MUL = "cuda/silu_mul"
SELECTED_RMS_NORM = "cuda/rms_norm"
SELECTED_ADD_RMS_NORM = "cuda/add_rms_norm"
SELECTED_GEMM_SWIGLU = "cuda/gemm_swiglu"
SELECTED_PAGED_ATTENTION = "cuda/paged_attention_decode"


def _contiguous(tensor: Any) -> Any:
    return tensor if tensor.is_contiguous() else tensor.contiguous()


def _in_place_operand(tensor: Any) -> Any:
    """The operand as rk_gemm_layout reads it: dense, or the transpose of a dense matrix."""
    if tensor.is_contiguous() or tensor.t().is_contiguous():
        return tensor
    return tensor.contiguous()


def _gemm_raw(a: Any, b: Any, output: Any | None) -> Any:
    ext = _native.extension()
    a, b = _in_place_operand(a), _in_place_operand(b)
    if output is None:
        return ext.gemm_views(a, b, None, 0)
    if output.is_contiguous():
        return ext.gemm_views(a, b, output, 0)
    output.copy_(ext.gemm_views(a, b, None, 0))
    return output


def _gemv_raw(x: Any, weight: Any) -> Any:
    if not weight.is_contiguous() and weight.t().is_contiguous():
        # weight is the transpose of a dense [K, N] matrix: x @ weight^T is the nn GEMM
        # x @ weight.t() on the stored matrix.
        return _native.extension().gemm_views(_contiguous(x), weight.t(), None, 0)
    return _native.extension().gemv(_contiguous(x), _contiguous(weight), 0)


def _autograd_functions() -> tuple[Any, Any]:
    import torch

    class _GemmFunction(torch.autograd.Function):
        @staticmethod
        def forward(ctx: Any, a: Any, b: Any) -> Any:
            ctx.save_for_backward(a, b)
            return _gemm_raw(a.detach(), b.detach(), None)

        @staticmethod
        def backward(ctx: Any, grad: Any) -> Any:
            a, b = ctx.saved_tensors
            grad = _contiguous(grad)
            # dA = dC @ B^T ("nt"), dB = A^T @ dC ("tn"): the saved operands are read
            # transposed in place.
            grad_a = _gemm_raw(grad, b.detach().t(), None) if ctx.needs_input_grad[0] else None
            grad_b = _gemm_raw(a.detach().t(), grad, None) if ctx.needs_input_grad[1] else None
            return grad_a, grad_b

    class _GemvFunction(torch.autograd.Function):
        @staticmethod
        def forward(ctx: Any, x: Any, weight: Any) -> Any:
            ctx.save_for_backward(x, weight)
            return _gemv_raw(x.detach(), weight.detach())

        @staticmethod
        def backward(ctx: Any, grad: Any) -> Any:
            x, weight = ctx.saved_tensors
            grad = _contiguous(grad)
            # out = x @ W^T:  dx = grad @ W,  dW = grad^T @ x
            grad_x = _gemm_raw(grad, weight.detach(), None) if ctx.needs_input_grad[0] else None
            grad_w = _gemm_raw(grad.t(), x.detach(), None) if ctx.needs_input_grad[1] else None
            return grad_x, grad_w

    return _GemmFunction, _GemvFunction


_FUNCTIONS: tuple[Any, Any] | None = None


def _functions() -> tuple[Any, Any]:
    global _FUNCTIONS
    if _FUNCTIONS is None:
        _FUNCTIONS = _autograd_functions()
    return _FUNCTIONS


def _needs_grad(torch_module: Any, *tensors: Any) -> bool:
    return torch_module.is_grad_enabled() and any(bool(t.requires_grad) for t in tensors)


def gemm(torch_module: Any, a: Any, b: Any, output: Any | None = None) -> Any:
    if _needs_grad(torch_module, a, b):
        if output is not None:
            raise RuntimeError("gemm(): an out= tensor does not support automatic differentiation")
        return _functions()[0].apply(a, b)
    return _gemm_raw(a, b, output)


def gemv(torch_module: Any, x: Any, weight: Any) -> Any:
    if _needs_grad(torch_module, x, weight):
        return _functions()[1].apply(x, weight)
    return _gemv_raw(x, weight)


# --------------------------------------------------------------- decode neighbours
# silu_mul / rms_norm / add_rms_norm (rk_silu_mul, rk_rms_norm, rk_add_rms_norm).  Their
# backward passes are not built yet: an input that requires gradients gets an autograd node
# whose backward raises, so a forward pass (e.g. evaluation with parameters that require
# gradients) still runs on these kernels and a backward pass fails loudly instead of
# silently computing with another library.

_NEIGHBOUR_FUNCTION: Any = None


def _no_backward_function() -> Any:
    global _NEIGHBOUR_FUNCTION
    if _NEIGHBOUR_FUNCTION is None:
        import torch

        class _ForwardOnly(torch.autograd.Function):
            @staticmethod
            def forward(ctx: Any, name: str, run: Any, *inputs: Any) -> Any:
                ctx.name = name
                return run(*[t.detach() for t in inputs])

            @staticmethod
            def backward(ctx: Any, *grads: Any) -> Any:
                raise NotImplementedError(f"{ctx.name}: the backward pass is not implemented in this build")

        _NEIGHBOUR_FUNCTION = _ForwardOnly
    return _NEIGHBOUR_FUNCTION


def _run(torch_module: Any, name: str, run: Any, *inputs: Any) -> Any:
    inputs = tuple(_contiguous(t) for t in inputs)
    if _needs_grad(torch_module, *inputs):
        return _no_backward_function().apply(name, run, *inputs)
    return run(*inputs)


def silu_mul(torch_module: Any, gate: Any, up: Any) -> Any:
    return _run(torch_module, "silu_mul", lambda g, u: _native.extension().silu_mul(g, u), gate, up)


def rms_norm(torch_module: Any, x: Any, weight: Any, eps: float) -> Any:
    return _run(torch_module, "rms_norm", lambda a, w: _native.extension().rms_norm(a, w, eps), x, weight)


def add_rms_norm(torch_module: Any, x: Any, residual: Any, weight: Any, eps: float) -> tuple[Any, Any]:
    out = _run(
        torch_module,
        "add_rms_norm",
        lambda a, r, w: tuple(_native.extension().add_rms_norm(a, r, w, eps)),
        x,
        residual,
        weight,
    )
    return out[0], out[1]


def _gemm_swiglu_raw(a: Any, b: Any) -> Any:
    ext = _native.extension()
    n = int(b.shape[1]) // 2
    try:
        return ext.gemm_swiglu(a, b, 0)
    except RuntimeError as error:
        if "variant does not support" not in str(error):
            raise
    # Shapes the fused kernel cannot take: this library's GEMM, then its silu_mul.
    y = ext.gemm(a, b, 0)
    return ext.silu_mul(y[:, :n].contiguous(), y[:, n:].contiguous())


def gemm_swiglu(torch_module: Any, a: Any, b: Any) -> Any:
    return _run(torch_module, "gemm_swiglu", _gemm_swiglu_raw, a, b)


def paged_attention_decode(
    torch_module: Any, query: Any, key_cache: Any, value_cache: Any, block_tables: Any, context_lengths: Any, scale: float
) -> Any:
    """rk_paged_attention_decode (inference only; the front-end rejects autograd inputs)."""

    return _native.extension().paged_attention_decode(query, key_cache, value_cache, block_tables, context_lengths, scale)
