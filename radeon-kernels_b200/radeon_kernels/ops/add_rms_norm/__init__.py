from radeon_kernels.ops.add_rms_norm.api import add_rms_norm

__all__ = ["add_rms_norm"]
