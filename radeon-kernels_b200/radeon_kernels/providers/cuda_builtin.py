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
SELECTED_SDPA = "cuda/sdpa"


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
# silu_mul / rms_norm / add_rms_norm (rk_silu_mul, rk_rms_norm, rk_add_rms_norm) and the
# fused gemm_swiglu.  Inputs that require gradients run the same forward kernels under an
# autograd node whose backward is this library's backward kernels (rk_silu_mul_backward,
# rk_rms_norm_backward, rk_add_rms_norm_backward): the gradients of the reference's fp32
# fallback graphs, which is what a reference user gets for such inputs.

_NEIGHBOUR_FUNCTIONS: dict[str, Any] | None = None


def _neighbour_functions() -> dict[str, Any]:
    global _NEIGHBOUR_FUNCTIONS
    if _NEIGHBOUR_FUNCTIONS is not None:
        return _NEIGHBOUR_FUNCTIONS
    import torch

    ext = _native.extension

    class _SiluMulFunction(torch.autograd.Function):
        @staticmethod
        def forward(ctx: Any, gate: Any, up: Any) -> Any:
            ctx.save_for_backward(gate, up)
            return ext().silu_mul(gate, up)

        @staticmethod
        def backward(ctx: Any, grad: Any) -> Any:
            gate, up = ctx.saved_tensors
            grad_gate, grad_up = ext().silu_mul_backward(_contiguous(grad), gate, up)
            return grad_gate, grad_up

    class _RmsNormFunction(torch.autograd.Function):
        @staticmethod
        def forward(ctx: Any, x: Any, weight: Any, eps: float) -> Any:
            ctx.save_for_backward(x, weight)
            ctx.eps = eps
            return ext().rms_norm(x, weight, eps)

        @staticmethod
        def backward(ctx: Any, grad: Any) -> Any:
            x, weight = ctx.saved_tensors
            grad_x, grad_w = ext().rms_norm_backward(_contiguous(grad), x, weight, ctx.eps, ctx.needs_input_grad[1])
            return grad_x, grad_w, None

    class _AddRmsNormFunction(torch.autograd.Function):
        @staticmethod
        def forward(ctx: Any, x: Any, residual: Any, weight: Any, eps: float) -> Any:
            out, residual_out = ext().add_rms_norm(x, residual, weight, eps)
            ctx.save_for_backward(residual_out, weight)
            ctx.eps = eps
            # An output that receives no gradient arrives as None, not as zeros: the
            # reference's graph adds no term for it (a -0 gradient stays -0).
            ctx.set_materialize_grads(False)
            return out, residual_out

        @staticmethod
        def backward(ctx: Any, grad_out: Any, grad_residual_out: Any) -> Any:
            residual_out, weight = ctx.saved_tensors
            if grad_out is None:
                # Only residual_out = x + residual carries a gradient: it passes to both.
                if grad_residual_out is None:
                    return None, None, None, None
                return grad_residual_out, grad_residual_out.clone(), None, None
            dres = None if grad_residual_out is None else _contiguous(grad_residual_out)
            grad_x, grad_residual, grad_w = ext().add_rms_norm_backward(
                _contiguous(grad_out), dres, residual_out, weight, ctx.eps, ctx.needs_input_grad[2]
            )
            return grad_x, grad_residual, grad_w, None

    class _GemmSwigluFunction(torch.autograd.Function):
        """Backward of the composition rk.gemm -> rk.silu_mul that the fused kernel replaces:
        the [M, 2N] product is recomputed (rounded, as the composition stores it), then
        silu_mul's backward and the two GEMM gradients (nt and tn layouts, read in place)."""

        @staticmethod
        def forward(ctx: Any, a: Any, b: Any) -> Any:
            ctx.save_for_backward(a, b)
            return _gemm_swiglu_raw(a, b)

        @staticmethod
        def backward(ctx: Any, grad: Any) -> Any:
            a, b = ctx.saved_tensors
            n = int(b.shape[1]) // 2
            y = _gemm_raw(a, b, None)
            grad_gate, grad_up = ext().silu_mul_backward(
                _contiguous(grad), y[:, :n].contiguous(), y[:, n:].contiguous()
            )
            grad_y = torch.cat([grad_gate, grad_up], dim=1)
            grad_a = _gemm_raw(grad_y, b.t(), None) if ctx.needs_input_grad[0] else None
            grad_b = _gemm_raw(a.t(), grad_y, None) if ctx.needs_input_grad[1] else None
            return grad_a, grad_b

    _NEIGHBOUR_FUNCTIONS = {
        "silu_mul": _SiluMulFunction,
        "rms_norm": _RmsNormFunction,
        "add_rms_norm": _AddRmsNormFunction,
        "gemm_swiglu": _GemmSwigluFunction,
    }
    return _NEIGHBOUR_FUNCTIONS


def silu_mul(torch_module: Any, gate: Any, up: Any) -> Any:
    gate, up = _contiguous(gate), _contiguous(up)
    if _needs_grad(torch_module, gate, up):
        return _neighbour_functions()["silu_mul"].apply(gate, up)
    return _native.extension().silu_mul(gate, up)


def rms_norm(torch_module: Any, x: Any, weight: Any, eps: float) -> Any:
    x, weight = _contiguous(x), _contiguous(weight)
    if _needs_grad(torch_module, x, weight):
        return _neighbour_functions()["rms_norm"].apply(x, weight, eps)
    return _native.extension().rms_norm(x, weight, eps)


def add_rms_norm(torch_module: Any, x: Any, residual: Any, weight: Any, eps: float) -> tuple[Any, Any]:
    x, residual, weight = _contiguous(x), _contiguous(residual), _contiguous(weight)
    if _needs_grad(torch_module, x, residual, weight):
        out, residual_out = _neighbour_functions()["add_rms_norm"].apply(x, residual, weight, eps)
    else:
        out, residual_out = _native.extension().add_rms_norm(x, residual, weight, eps)
    return out, residual_out


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
    a, b = _contiguous(a), _contiguous(b)
    if _needs_grad(torch_module, a, b):
        return _neighbour_functions()["gemm_swiglu"].apply(a, b)
    return _gemm_swiglu_raw(a, b)


def paged_attention_decode(
    torch_module: Any, query: Any, key_cache: Any, value_cache: Any, block_tables: Any, context_lengths: Any, scale: float
) -> Any:
    """rk_paged_attention_decode (inference only; the front-end rejects autograd inputs)."""

    return _native.extension().paged_attention_decode(query, key_cache, value_cache, block_tables, context_lengths, scale)


def sdpa(torch_module: Any, query: Any, key: Any, value: Any, is_causal: bool, scale: float) -> Any:
    """rk_sdpa (inference only; the front-end rejects autograd and non-contiguous inputs)."""

    return _native.extension().sdpa(query, key, value, is_causal, scale)
