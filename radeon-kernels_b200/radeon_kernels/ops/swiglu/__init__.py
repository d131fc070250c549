from radeon_kernels.ops.swiglu.api import silu_mul

__all__ = ["silu_mul"]
