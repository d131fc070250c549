from radeon_kernels.ops.gemv.api import gemv

__all__ = ["gemv"]
