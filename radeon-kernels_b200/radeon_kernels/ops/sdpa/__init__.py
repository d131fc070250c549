from radeon_kernels.ops.sdpa.api import sdpa

__all__ = ["sdpa"]
