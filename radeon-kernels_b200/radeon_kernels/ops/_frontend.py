"""Operator front-ends as checked argument bundles.

A public operator binds its arguments by name into an :class:`Args` bundle and states its
rules as a short sequence of checks on it -- tensor kinds and ranks, groups that must share
device and dtype, and shape predicates with the message to raise -- then builds its
dispatch signature and hands everything to the operator runtime with :func:`dispatch`.
Every message is prefixed with the operator name, so the rules read as what they check.

The checks raise what the reference's front-ends raise, in the same order, so callers and
tests that match the messages keep working: ``TypeError`` for a non-tensor, a wrong dtype
or index dtype and a wrong scalar type, ``ValueError`` for rank, device, shape and value
errors -- all before anything is dispatched or recorded.
"""

from __future__ import annotations

import math
from typing import Any, Callable, Mapping, Sequence

from radeon_kernels.ops._common import (
    TensorContext,
    index_dtype_name,
    tensor_context,
    validate_eps,
    validate_index_tensor,
    validate_same,
    validate_tensor,
)


class Args:
    """Named arguments of one call of ``operator`` plus the checks that apply to them."""

    def __init__(self, operator: str, torch_module: Any, **values: Any) -> None:
        self.operator = operator
        self.torch = torch_module
        self.values = values

    def __getitem__(self, name: str) -> Any:
        return self.values[name]

    # -- kinds -----------------------------------------------------------------------
    def tensors(self, **ranks: int) -> Args:
        """fp16/bf16 CUDA tensors of the given ranks, checked in the order given."""

        for name, rank in ranks.items():
            validate_tensor(self.torch, self.values[name], name=name, rank=rank, operator=self.operator)
        return self

    def indices(self, **ranks: int) -> Args:
        """int32/int64 CUDA tensors of the given ranks."""

        for name, rank in ranks.items():
            validate_index_tensor(self.torch, self.values[name], name=name, rank=rank, operator=self.operator)
        return self

    def alike(self, *names: str) -> Args:
        """Each named tensor shares device and dtype with the one before it."""

        for first, second in zip(names, names[1:]):
            validate_same(self.operator, self.values[first], self.values[second], first_name=first, second_name=second)
        return self

    # -- rules -----------------------------------------------------------------------
    def expect(self, holds: bool, message: str, error: type[Exception] = ValueError) -> Args:
        if not holds:
            raise error(f"{self.operator} {message}")
        return self

    def dims(self, name: str) -> tuple[int, ...]:
        return tuple(int(size) for size in self.values[name].shape)

    def context(self, *names: str) -> TensorContext:
        return tensor_context(self.torch, self.operator, *(self.values[name] for name in names))

    def inference_only(self, *names: str) -> TensorContext:
        """Context of the named tensors, which must be contiguous and need no gradient."""

        context = self.context(*names)
        self.expect(context.contiguous, "inputs must be contiguous")
        self.expect(not context.requires_grad, "is inference-only and does not support autograd")
        return context

    # -- scalars ---------------------------------------------------------------------
    def eps(self, value: Any) -> float:
        return validate_eps(value, self.operator)

    def scale(self, value: Any, head_dim: int) -> tuple[float, str]:
        """(softmax scale, "default" | "explicit"); None means 1/sqrt(head_dim)."""

        if value is None:
            return 1.0 / math.sqrt(head_dim), "default"
        self.expect(not isinstance(value, bool) and isinstance(value, (int, float)), "scale must be a number", TypeError)
        scale = float(value)
        self.expect(math.isfinite(scale) and scale > 0, "scale must be positive and finite")
        return scale, "explicit"

    def index_dtype(self, name: str) -> str:
        return index_dtype_name(self.torch, self.values[name].dtype, self.operator)


def dispatch(
    args: Args,
    runtime: Any,
    *,
    semantic_version: str,
    signature: Mapping[str, Any],
    device_index: int,
    native_arguments: Sequence[Any],
    fallback: Callable[..., Any],
    fallback_selected: str,
) -> Any:
    """Runs the operator through the dispatch runtime; ``fallback(torch, *native_arguments)``
    is this library's kernel for calls no pack entry serves."""

    arguments = tuple(native_arguments)
    return runtime.execute(
        operator=args.operator,
        semantic_version=semantic_version,
        signature=dict(signature),
        device_index=device_index,
        torch_module=args.torch,
        native_arguments=arguments,
        fallback=lambda: fallback(args.torch, *arguments),
        fallback_selected=fallback_selected,
    )


__all__ = ["Args", "dispatch"]
