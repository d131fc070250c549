"""rk_gemv_fixed_scratch -- the GEMV entry point that allocates nothing.

It exists for callers that cannot give the library device memory: plugins hosted by
an engine that owns every device allocation and hands a custom op only its inputs and
outputs, and serving loops that must not call cudaMalloc on the hot path.  It runs the
stream-K tensor-core GEMV, whose split-K scratch is a fixed array inside the library.
Here it is checked, through the C ABI, against the existing entry point rk_gemv_ex on
two calls in a row: the second call must still be right although the array keeps the
first call's contents.  Collected last on purpose, and self-contained so it also passes alone in a
fresh process.
"""

from __future__ import annotations

import ctypes

import pytest

from gpu_util import seeded, to_bits
from oracle import oracle
from radeon_kernels import _native

pytestmark = pytest.mark.gpu


def _stream():
    import torch

    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize(
    "dtype, m, n, k",
    [("bf16", 5, 8192, 8192), ("fp16", 16, 4096, 14336), ("bf16", 32, 1000, 4104), ("fp16", 3, 40000, 512)],
)
def test_fixed_scratch_matches_the_workspace_entry_point(dtype, m, n, k):
    import torch

    lib = _native.library()
    code = _native.RK_DTYPE_BF16 if dtype == "bf16" else _native.RK_DTYPE_FP16
    gen = torch.Generator().manual_seed(m * 131 + n)
    x = seeded((m, k), 21, "normal", dtype, gen).cuda()
    w = seeded((n, k), 21, f"normal/{k}", dtype, gen).cuda()

    need = ctypes.c_size_t(0)
    assert lib.rk_gemv_workspace_size(m, n, k, code, _native.GEMV_VARIANTS["tc"], ctypes.byref(need)) == 0
    workspace = torch.zeros(max(need.value, 1), dtype=torch.uint8, device="cuda")
    ref = torch.empty(m, n, dtype=x.dtype, device="cuda")
    st = lib.rk_gemv_ex(
        ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(ref.data_ptr()),
        m, n, k, code, _native.GEMV_VARIANTS["tc"], ctypes.c_void_p(workspace.data_ptr()), need.value, _stream(),
    )
    assert st == _native.RK_OK, _native.status_text(st)

    for _ in range(2):
        out = torch.full((m, n), float("nan"), dtype=x.dtype, device="cuda")
        st = lib.rk_gemv_fixed_scratch(
            ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(out.data_ptr()),
            m, n, k, code, _stream(),
        )
        assert st == _native.RK_OK, _native.status_text(st)
        torch.cuda.synchronize()
        assert oracle.parity_error(oracle.widen(to_bits(out), dtype), oracle.widen(to_bits(ref), dtype)) <= oracle.TOLERANCE[dtype]
    assert lib.rk_device_status(_stream()) == _native.RK_OK


def test_fixed_scratch_rejects_bad_arguments():
    import torch

    lib = _native.library()
    x = torch.zeros(33, 64, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(64, 64, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(33, 64, dtype=torch.bfloat16, device="cuda")
    args = (ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(out.data_ptr()))
    assert lib.rk_gemv_fixed_scratch(*args, 33, 64, 64, 1, _stream()) == _native.RK_ERR_INVALID_ARGUMENT
    assert lib.rk_gemv_fixed_scratch(*args, 1, 64, 60, 1, _stream()) == _native.RK_ERR_UNSUPPORTED  # K % 8
