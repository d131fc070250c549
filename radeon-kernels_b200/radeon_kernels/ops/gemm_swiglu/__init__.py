from radeon_kernels.ops.gemm_swiglu.api import gemm_swiglu

__all__ = ["gemm_swiglu"]
