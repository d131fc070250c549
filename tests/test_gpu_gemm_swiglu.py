"""Fused FFN-up + SwiGLU (rk_gemm_swiglu / rk.gemm_swiglu) on a B200.

Definition (no counterpart in the reference): silu(A @ B[:, :N]) * (A @ B[:, N:]) from the
fp32 sums, rounded once -- the reference's GEMM and silu_mul composed in fp32
(oracle.gemm_swiglu).  Gate: the GEMM parity rule (oracle.assert_parity), since both products
are long fp32 sums whose order differs.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from gpu_util import DTYPE_CODE, device_status, seeded, stream_handle, to_bits, torch_dtype
from oracle import oracle
from radeon_kernels import _native

pytestmark = pytest.mark.gpu
GEMM = _native.GEMM_VARIANTS
SENTINEL = 0x7E7E


def swiglu_abi(a, b, c, variant, dtype):
    m, k = a.shape
    n = c.shape[1]
    return _native.library().rk_gemm_swiglu(
        ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(b.data_ptr()), ctypes.c_void_p(c.data_ptr()),
        m, n, k, DTYPE_CODE[dtype], variant, stream_handle(),
    )


def _guarded(torch, rows, cols, dtype, pad=4096):
    buf = torch.full((rows * cols + 2 * pad,), SENTINEL, dtype=torch.int16, device="cuda")
    return buf, buf.view(torch_dtype(dtype))[pad : pad + rows * cols].view(rows, cols)


def _intact(buf, pad=4096):
    bits = to_bits(buf)
    return bool(np.all(bits[:pad] == SENTINEL) and np.all(bits[-pad:] == SENTINEL))


@pytest.mark.parametrize("variant", ["auto", "tc_1sm", "tc_2sm"])
@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize(
    "m, n, k",
    [(256, 512, 1024), (300, 200, 1000), (64, 8, 64), (1, 128, 8), (513, 136, 264)],
)
def test_matches_the_fp32_composition(m, n, k, dtype, variant):
    import torch

    gen = torch.Generator().manual_seed(m + n + k)
    a = seeded((m, k), 0, "normal", dtype, gen)
    b = seeded((k, 2 * n), 0, f"normal/{k}", dtype, gen)
    buf, c = _guarded(torch, m, n, dtype)
    ad, bd = a.cuda(), b.cuda()
    assert swiglu_abi(ad, bd, c, GEMM[variant], dtype) == _native.RK_OK
    again = torch.empty_like(c)
    assert swiglu_abi(ad, bd, again, GEMM[variant], dtype) == _native.RK_OK
    torch.cuda.synchronize()
    assert device_status() == _native.RK_OK
    assert _intact(buf)
    assert torch.equal(c.view(torch.int16), again.view(torch.int16))
    ref_bits, ref32 = oracle.gemm_swiglu(to_bits(a), to_bits(b), dtype)
    oracle.assert_parity(to_bits(c), ref_bits, ref32, dtype)


def test_ffn_up_config4_full_size():
    """BASELINE config 4's FFN-up shape with the gate/up pair: A [4096, 4096], B [4096, 28672]."""

    import torch

    m, n, k, dtype = 4096, 14336, 4096, "fp16"
    gen = torch.Generator(device="cuda").manual_seed(3)
    a = (torch.randn((m, k), generator=gen, device="cuda") / 64).half()
    b = (torch.randn((k, 2 * n), generator=gen, device="cuda") / 64).half()
    c = torch.empty(m, n, dtype=torch.float16, device="cuda")
    assert swiglu_abi(a, b, c, GEMM["auto"], dtype) == _native.RK_OK
    # Test-side check of every element: the fp32 product (cuBLAS, test infrastructure only)
    # composed with silu in fp32.
    y = torch.mm(a.float(), b.float())
    g, u = y[:, :n], y[:, n:]
    ref32 = g * torch.sigmoid(g) * u
    torch.cuda.synchronize()
    err = ((c.float() - ref32).abs().max() / ref32.abs().max()).item()
    assert err <= oracle.TOLERANCE[dtype], err
    # and the C oracle on sampled rows
    rows = [0, 1, 2047, 4095]
    sub_bits, sub32 = oracle.gemm_swiglu(to_bits(a[rows]), to_bits(b), dtype)
    oracle.assert_parity(to_bits(c[rows]), sub_bits, sub32, dtype)


def test_unsupported_shapes_are_refused_and_the_api_composes():
    import torch

    import radeon_kernels as rk
    from radeon_kernels.ops._runtime import reset_operator_runtime

    reset_operator_runtime()
    gen = torch.Generator().manual_seed(9)
    a = seeded((33, 64), 0, "normal", "bf16", gen)
    b = seeded((64, 24), 0, "normal/64", "bf16", gen)  # N = 12: not a multiple of 8
    c = torch.empty(33, 12, dtype=torch.bfloat16, device="cuda")
    assert swiglu_abi(a.cuda(), b.cuda(), c, GEMM["auto"], "bf16") == _native.RK_ERR_UNSUPPORTED
    out = rk.gemm_swiglu(a.cuda(), b.cuda())
    record = rk.get_last_dispatch()
    assert record["selected"] in ("native/gemm_swiglu", "cuda/gemm_swiglu"), record["reason"]
    # The composed path is the reference's own two-operator FFN: the [M, 2N] product is
    # rounded to the dtype, then silu_mul runs on it.  Its oracle is that composition.
    y_bits, y32 = oracle.gemm(to_bits(a), to_bits(b), "bf16")
    silu_bits, silu32 = oracle.silu_mul(y_bits[:, :12], y_bits[:, 12:], "bf16")
    oracle.assert_parity(to_bits(out), silu_bits, silu32, "bf16")


def test_public_api_dispatches_to_the_fused_kernel():
    import torch

    import radeon_kernels as rk
    from radeon_kernels.ops._runtime import reset_operator_runtime

    reset_operator_runtime()
    gen = torch.Generator().manual_seed(10)
    a = seeded((128, 512), 0, "normal", "fp16", gen).cuda()
    b = seeded((512, 1024), 0, "normal/512", "fp16", gen).cuda()
    out = rk.gemm_swiglu(a, b)
    record = rk.get_last_dispatch()
    assert record["operator"] == "gemm_swiglu"
    assert record["selected"] == "native/gemm_swiglu", record["reason"]
    ref_bits, ref32 = oracle.gemm_swiglu(to_bits(a), to_bits(b), "fp16")
    oracle.assert_parity(to_bits(out), ref_bits, ref32, "fp16")
