"""rk_gemv_fixed_scratch -- the GEMV entry point that allocates nothing.

It exists for callers that cannot give the library device memory: plugins hosted by
an engine that owns every device allocation and hands a custom op only its inputs and
outputs, and serving loops that must not call cudaMalloc on the hot path.  It runs the
stream-K tensor-core GEMV, whose split-K scratch is a fixed array inside the library.

Checked through the C ABI on two calls in a row (the second must still be right although
the array keeps the first call's contents): against the C oracle on the same CPU inputs,
against the existing entry point rk_gemv_ex (cluster split-K: a different reduction,
so a real cross-check), and -- through rk_debug_last_kernel -- that the stream-K kernel is
the one that ran.  One case starts from an array filled with garbage, as an interrupted
call could leave it: the entry point must clear its tickets itself.  Collected last on
purpose, and self-contained so it also passes alone in a fresh process.
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


def _fixed(lib, x, w, out, m, n, k, code):
    return lib.rk_gemv_fixed_scratch(
        ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(out.data_ptr()),
        m, n, k, code, _stream(),
    )


@pytest.mark.parametrize("dirty", [False, True], ids=["clean", "garbage-filled"])
@pytest.mark.parametrize(
    "dtype, m, n, k",
    [("bf16", 5, 8192, 8192), ("fp16", 16, 4096, 14336), ("bf16", 32, 1000, 4104), ("fp16", 3, 40000, 512)],
)
def test_fixed_scratch_matches_the_oracle_and_the_workspace_entry_point(dtype, m, n, k, dirty):
    import torch

    lib = _native.library()
    lib.rk_gemv_tc_set_cluster(0)  # the built-in strategy for rk_gemv_ex, whatever ran before
    code = _native.RK_DTYPE_BF16 if dtype == "bf16" else _native.RK_DTYPE_FP16
    gen = torch.Generator().manual_seed(m * 131 + n)
    x_cpu = seeded((m, k), 21, "normal", dtype, gen)
    w_cpu = seeded((n, k), 21, f"normal/{k}", dtype, gen)
    x, w = x_cpu.cuda(), w_cpu.cuda()
    o_bits, o32 = oracle.gemv(to_bits(x_cpu), to_bits(w_cpu), dtype)

    need = ctypes.c_size_t(0)
    assert lib.rk_gemv_workspace_size(m, n, k, code, _native.GEMV_VARIANTS["tc"], ctypes.byref(need)) == 0
    workspace = torch.zeros(max(need.value, 1), dtype=torch.uint8, device="cuda")
    ref = torch.empty(m, n, dtype=x.dtype, device="cuda")
    st = lib.rk_gemv_ex(
        ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(ref.data_ptr()),
        m, n, k, code, _native.GEMV_VARIANTS["tc"], ctypes.c_void_p(workspace.data_ptr()), need.value, _stream(),
    )
    assert st == _native.RK_OK, _native.status_text(st)
    # Cluster split-K, in either exchange form (pulled, or pushed into the leader CTA).
    assert lib.rk_debug_last_kernel() in (b"gemv_tc_kernel", b"gemv_tc_kernel<push>")

    if dirty:
        assert lib.rk_debug_fill_fixed_scratch(0xA7, _stream()) == _native.RK_OK
    for _ in range(2):
        out = torch.full((m, n), float("nan"), dtype=x.dtype, device="cuda")
        st = _fixed(lib, x, w, out, m, n, k, code)
        assert st == _native.RK_OK, _native.status_text(st)
        assert lib.rk_debug_last_kernel() == b"gemv_tc_sk_kernel"
        torch.cuda.synchronize()
        oracle.assert_parity(to_bits(out), o_bits, o32, dtype)
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
    # Taller than the ticket prefix covers (16384 tiles of 128 rows): rejected before any
    # memory is touched, so the small buffers here are never read.
    assert lib.rk_gemv_fixed_scratch(*args, 1, 2_097_152 + 1, 64, 1, _stream()) == _native.RK_ERR_TOO_LARGE
