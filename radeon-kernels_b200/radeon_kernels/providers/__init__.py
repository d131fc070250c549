"""Provider adapters: ``native`` (a published pack winner) and ``cuda`` (built-in kernels)."""

from radeon_kernels.providers.native import NativeProviderError

__all__ = ["NativeProviderError"]
