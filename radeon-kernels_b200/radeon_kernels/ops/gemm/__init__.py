from radeon_kernels.ops.gemm.api import GemmDispatchError, GemmRuntime, gemm, reset_runtime

__all__ = ["GemmDispatchError", "GemmRuntime", "gemm", "reset_runtime"]
