"""B200 (sm_100a) dense-contraction kernels with the radeon-kernels public API.

``gemm(a, b, *, out=None)`` and ``gemv(x, weight)`` dispatch through the static manifests
in ``dispatch/`` to the built-in sm_100a kernel pack, and fall back to the same library's
generic CUDA kernels; ``explain_last_dispatch()`` / ``get_last_dispatch()`` report what ran.
"""

from radeon_kernels.ops.gemm import gemm
from radeon_kernels.ops.gemv import gemv
from radeon_kernels.runtime.explain import explain_last_dispatch, get_last_dispatch

__version__ = "0.1.0"

__all__ = ["__version__", "explain_last_dispatch", "gemm", "gemv", "get_last_dispatch"]
