"""Calls into a verified pack entrypoint, with the reference's safety checks.

Same contract as src/radeon_kernels/providers/native.py:14-53: only the ``native``
provider is accepted; a GEMM launch must be exactly ``{"variant": int >= 0}`` and the
entrypoint must write into and return the caller's output tensor; a generic entrypoint is
called as ``entry(*arguments, **launch)`` and must return something.
"""

from __future__ import annotations

from typing import Any, Mapping

from radeon_kernels.errors import RadeonKernelsError
from radeon_kernels.runtime.loader import PrecompiledArtifactLoader
from radeon_kernels.runtime.registry import ArtifactSpec


class NativeProviderError(RadeonKernelsError):
    """An approved native launch cannot be executed safely."""


def execute(
    loader: PrecompiledArtifactLoader,
    artifact: ArtifactSpec,
    launch: Mapping[str, str | int | float | bool],
    *arguments: Any,
) -> Any:
    if artifact.provider != "native":
        raise NativeProviderError(f"unsupported native winner provider: {artifact.provider!r}")
    result = loader.load_entrypoint(artifact).callable(*arguments, **dict(launch))
    if result is None:
        raise NativeProviderError("native entrypoint returned no output")
    return result


def gemm(
    loader: PrecompiledArtifactLoader,
    artifact: ArtifactSpec,
    launch: Mapping[str, str | int | float | bool],
    a: Any,
    b: Any,
    output: Any,
) -> Any:
    if artifact.provider != "native":
        raise NativeProviderError(f"unsupported GEMM winner provider: {artifact.provider!r}")
    if set(launch) != {"variant"}:
        raise NativeProviderError("native GEMM launch must contain exactly one variant")
    variant = launch["variant"]
    if isinstance(variant, bool) or not isinstance(variant, int) or variant < 0:
        raise NativeProviderError("native GEMM variant must be a non-negative integer")
    result = loader.load_entrypoint(artifact).callable(a, b, output, variant)
    if result is None:
        raise NativeProviderError("native GEMM returned no output tensor")
    if hasattr(result, "data_ptr") and result.data_ptr() != output.data_ptr():
        raise NativeProviderError("native GEMM did not return the caller-provided output")
    return result
