"""Device-side failure detection without a GPU fault.

The tensor-core GEMM's MMA role is made to wait on an mbarrier nothing arrives on (host
test hook).  Its bounded wait must run out, every role must drain and exit, the kernel
must report RK_ERR_TIMEOUT through the status word, and the context must stay usable.
"""

from __future__ import annotations

import pytest

from gpu_util import abi_gemm, device_status, seeded, to_bits
from oracle import oracle
from radeon_kernels import _native

pytestmark = pytest.mark.gpu


def test_stalled_pipeline_reports_timeout_and_context_survives():
    import torch

    lib = _native.library()
    a = seeded((256, 128), 0, "uniform", "bf16").cuda()
    b = seeded((128, 512), 1, "uniform", "bf16").cuda()
    c = torch.zeros(256, 512, dtype=torch.bfloat16, device="cuda")
    assert device_status() == _native.RK_OK
    lib.rk_set_wait_timeout_ns(50_000_000)  # 50 ms per wait
    try:
        lib.rk_debug_inject_stall(1)
        assert abi_gemm(a, b, c, _native.GEMM_VARIANTS["tc_1sm"], "bf16") == _native.RK_OK
        torch.cuda.synchronize()  # the kernel returned on its own
        assert device_status() == _native.RK_ERR_TIMEOUT
        assert device_status() == _native.RK_OK  # read-and-clear
    finally:
        lib.rk_debug_inject_stall(0)
        lib.rk_set_wait_timeout_ns(0)
    # the same context still computes correct results
    assert abi_gemm(a, b, c, _native.GEMM_VARIANTS["tc_1sm"], "bf16") == _native.RK_OK
    torch.cuda.synchronize()
    assert device_status() == _native.RK_OK
    ref_bits, ref32 = oracle.gemm(to_bits(a), to_bits(b), "bf16")
    oracle.assert_parity(to_bits(c), ref_bits, ref32, "bf16")
