"""Calls into a verified pack entrypoint, with the reference's safety checks.

Contract of src/radeon_kernels/providers/native.py:14-53: only the ``native`` provider runs;
a GEMM launch is exactly ``{"variant": int >= 0}`` and the entrypoint must write into and
return the caller's output tensor; any other entrypoint is called as
``entry(*arguments, **launch)`` and must return something.  Each check raises
:class:`NativeProviderError`, which the operator runtime turns into its fallback.
"""

from __future__ import annotations

from typing import Any, Callable, Mapping

from radeon_kernels.errors import RadeonKernelsError
from radeon_kernels.runtime.loader import PrecompiledArtifactLoader
from radeon_kernels.runtime.registry import ArtifactSpec

Launch = Mapping[str, "str | int | float | bool"]


class NativeProviderError(RadeonKernelsError):
    """An approved native launch cannot be executed safely."""


def _entrypoint(loader: PrecompiledArtifactLoader, artifact: ArtifactSpec, role: str) -> Callable[..., Any]:
    if artifact.provider != "native":
        raise NativeProviderError(f"unsupported {role} provider: {artifact.provider!r}")
    return loader.load_entrypoint(artifact).callable


def _gemm_variant(launch: Launch) -> int:
    if set(launch) != {"variant"}:
        raise NativeProviderError("native GEMM launch must contain exactly one variant")
    variant = launch["variant"]
    if type(variant) is not int or variant < 0:
        raise NativeProviderError("native GEMM variant must be a non-negative integer")
    return variant


def execute(loader: PrecompiledArtifactLoader, artifact: ArtifactSpec, launch: Launch, *arguments: Any) -> Any:
    result = _entrypoint(loader, artifact, "native winner")(*arguments, **dict(launch))
    if result is None:
        raise NativeProviderError("native entrypoint returned no output")
    return result


def gemm(loader: PrecompiledArtifactLoader, artifact: ArtifactSpec, launch: Launch, a: Any, b: Any, output: Any) -> Any:
    if artifact.provider != "native":  # checked before the launch, as the reference orders it
        raise NativeProviderError(f"unsupported GEMM winner provider: {artifact.provider!r}")
    variant = _gemm_variant(launch)
    result = _entrypoint(loader, artifact, "GEMM winner")(a, b, output, variant)
    if result is None:
        raise NativeProviderError("native GEMM returned no output tensor")
    if hasattr(result, "data_ptr") and result.data_ptr() != output.data_ptr():
        raise NativeProviderError("native GEMM did not return the caller-provided output")
    return result
