from radeon_kernels.ops.paged_attention.api import paged_attention_decode

__all__ = ["paged_attention_decode"]
