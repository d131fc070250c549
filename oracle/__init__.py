"""CPU oracle for the GEMM/GEMV hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may
import this package, and only as the checker / the timed reference arm.  The product
(``radeon-kernels_b200/``) never imports it and has no CPU path.
"""
