from radeon_kernels.ops.rms_norm.api import rms_norm

__all__ = ["rms_norm"]
