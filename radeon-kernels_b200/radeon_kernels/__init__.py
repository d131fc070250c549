"""B200 (sm_100a) dense-contraction kernels with the radeon-kernels public API.

``gemm(a, b, *, out=None)`` and ``gemv(x, weight)`` -- and their decode-time neighbours
``silu_mul(gate, up)``, ``rms_norm(x, weight, eps)``, ``add_rms_norm(x, residual, weight,
eps)``, the fused FFN-up ``gemm_swiglu(a, w_gate_up)``, ``paged_attention_decode`` and
``sdpa`` --
dispatch through the static manifests in ``dispatch/`` to the built-in sm_100a
kernel pack, and fall back to the same library's CUDA kernels; ``explain_last_dispatch()`` /
``get_last_dispatch()`` report what ran.
"""

from radeon_kernels.ops.add_rms_norm import add_rms_norm
from radeon_kernels.ops.gemm import gemm
from radeon_kernels.ops.gemm_swiglu import gemm_swiglu
from radeon_kernels.ops.gemv import gemv
from radeon_kernels.ops.paged_attention import paged_attention_decode
from radeon_kernels.ops.rms_norm import rms_norm
from radeon_kernels.ops.sdpa import sdpa
from radeon_kernels.ops.swiglu import silu_mul
from radeon_kernels.runtime.explain import explain_last_dispatch, get_last_dispatch

__version__ = "0.1.0"

__all__ = [
    "__version__",
    "add_rms_norm",
    "explain_last_dispatch",
    "gemm",
    "gemm_swiglu",
    "gemv",
    "get_last_dispatch",
    "paged_attention_decode",
    "rms_norm",
    "sdpa",
    "silu_mul",
]
