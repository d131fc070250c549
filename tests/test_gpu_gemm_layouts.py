"""Transposed operand layouts (rk_gemm_layout; "nt"/"tn" of the reference's Layout enum,
src/radeon_kernels/ops/gemm/spec.py:12-15) against the oracle, and the autograd paths that
use them.

Each case stores A as [M,K] ("n") or [K,M] ("t") and B as [K,N] ("n") or [N,K] ("t"), runs
every variant through the C ABI, and checks the product with the GEMM parity gate against
the C oracle fed the logical (materialised) operands.  Outputs land inside a sentinel guard.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from gpu_util import abi_gemm_layout, device_status, seeded, to_bits, torch_dtype
from oracle import oracle
from radeon_kernels import _native

pytestmark = pytest.mark.gpu
GEMM = _native.GEMM_VARIANTS
SENTINEL = 0x7E7E
LAYOUTS = ["nn", "nt", "tn", "tt"]
SHAPES = [
    (128, 256, 64),
    (256, 512, 128),
    (200, 264, 72),  # M, N not multiples of the tile: TMA zero fill + predicated stores
    (8, 8, 8),
    (520, 1032, 1000),
    (1024, 1024, 1024),
    (12, 40, 24),  # M % 8 != 0: a transposed A (row stride 12) takes the generic kernel
    (3, 17, 9),  # generic kernel only
]


def _tc_ok(layout, m, n, k):
    return n % 8 == 0 and k % 8 == 0 and (layout[0] == "n" or m % 8 == 0)


def _guarded(torch, rows, cols, dtype, pad=4096):
    buf = torch.full((rows * cols + 2 * pad,), SENTINEL, dtype=torch.int16, device="cuda").view(torch_dtype(dtype))
    return buf, buf[pad : pad + rows * cols].view(rows, cols)


def _guards_intact(buf, pad=4096):
    bits = to_bits(buf)
    return bool(np.all(bits[:pad] == SENTINEL) and np.all(bits[-pad:] == SENTINEL))


def _operands(layout, m, n, k, dtype):
    import torch

    gen = torch.Generator().manual_seed(m * 31 + n * 7 + k + LAYOUTS.index(layout))
    a = seeded((m, k), 0, "uniform", dtype, gen)
    b = seeded((k, n), 0, "uniform", dtype, gen)
    a_stored = a.t().contiguous() if layout[0] == "t" else a
    b_stored = b.t().contiguous() if layout[1] == "t" else b
    return a, b, a_stored, b_stored


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("layout", LAYOUTS)
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_layouts_against_oracle(shape, layout, dtype):
    import torch

    m, n, k = shape
    a, b, a_stored, b_stored = _operands(layout, m, n, k, dtype)
    c_bits, c32 = oracle.gemm(to_bits(a), to_bits(b), dtype)
    a_dev, b_dev = a_stored.cuda(), b_stored.cuda()
    a_before, b_before = to_bits(a_dev), to_bits(b_dev)
    for variant in ("auto", "tc_1sm", "tc_2sm", "simt"):
        buf, c = _guarded(torch, m, n, dtype)
        status = abi_gemm_layout(a_dev, b_dev, c, layout, GEMM[variant], dtype)
        if variant in ("tc_1sm", "tc_2sm") and not _tc_ok(layout, m, n, k):
            assert status == _native.RK_ERR_UNSUPPORTED, variant
            continue
        assert status == _native.RK_OK, (variant, _native.status_text(status))
        torch.cuda.synchronize()
        assert device_status() == _native.RK_OK
        assert _guards_intact(buf), f"{variant} wrote outside C"
        oracle.assert_parity(to_bits(c), c_bits, c32, dtype)
    assert np.array_equal(to_bits(a_dev), a_before) and np.array_equal(to_bits(b_dev), b_before)


@pytest.mark.parametrize("layout", ["nt", "tn"])
def test_config4_shape_transposed(layout):
    """BASELINE config 4's shape (4096 x 14336 x 4096 fp16) with one operand stored transposed:
    full fp32 check on the GPU plus the C oracle on sampled rows."""

    import torch

    m, n, k = 4096, 14336, 4096
    gen = torch.Generator().manual_seed(3)
    a = (torch.randn((m, k), generator=gen) / 64).to(torch.float16)
    b = (torch.randn((k, n), generator=gen) / 64).to(torch.float16)
    a_dev, b_dev = a.cuda(), b.cuda()
    a_stored = a_dev.t().contiguous() if layout[0] == "t" else a_dev
    b_stored = b_dev.t().contiguous() if layout[1] == "t" else b_dev
    c = torch.empty(m, n, dtype=torch.float16, device="cuda")
    assert abi_gemm_layout(a_stored, b_stored, c, layout, GEMM["auto"], "fp16") == _native.RK_OK
    torch.cuda.synchronize()
    assert device_status() == _native.RK_OK
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref32 = torch.mm(a_dev.float(), b_dev.float())
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    err = (c.float() - ref32).abs().max().item() / ref32.abs().max().item()
    assert err <= oracle.TOLERANCE["fp16"], err
    rows = np.array([0, 1, 777, 2048, 4095])
    o_bits, o32 = oracle.gemm(to_bits(a[rows]), to_bits(b), "fp16")
    oracle.assert_parity(to_bits(c[rows]), o_bits, o32, "fp16")


def test_binding_reads_transposed_views_in_place():
    """gemm_views takes x.t() views without a copy and matches the oracle."""

    import torch

    ext = _native.extension()
    a, b, a_t, b_t = _operands("tt", 256, 384, 192, "bf16")
    a_dev, b_dev = a_t.cuda().t(), b_t.cuda().t()  # transposed views of dense storage
    assert not a_dev.is_contiguous() and not b_dev.is_contiguous()
    c = ext.gemm_views(a_dev, b_dev, None, 0)
    c_bits, c32 = oracle.gemm(to_bits(a), to_bits(b), "bf16")
    oracle.assert_parity(to_bits(c), c_bits, c32, "bf16")
    out = torch.empty(256, 384, dtype=torch.bfloat16, device="cuda")
    assert ext.gemm_views(a.cuda(), b_dev, out, 0).data_ptr() == out.data_ptr()
    oracle.assert_parity(to_bits(out), c_bits, c32, "bf16")
    with pytest.raises(RuntimeError, match="dense matrices"):
        ext.gemm_views(a.cuda()[:, ::2], b.cuda()[::2, :], None, 0)


def test_public_gemm_on_transposed_views():
    """rk.gemm(a, b.t()): the signature says contiguous=False, no manifest entry matches, and the
    built-in cuda provider runs the nt layout; the result matches the oracle."""

    import radeon_kernels as rk

    a, b, _, b_stored = _operands("nt", 128, 256, 64, "fp16")
    c = rk.gemm(a.cuda(), b_stored.cuda().t())
    assert rk.get_last_dispatch()["selected"] == "cuda/gemm"
    c_bits, c32 = oracle.gemm(to_bits(a), to_bits(b), "fp16")
    oracle.assert_parity(to_bits(c), c_bits, c32, "fp16")


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_gemm_backward_uses_transposed_layouts(dtype):
    """dA = dC @ B^T and dB = A^T @ dC, each against the oracle's GEMM of the materialised
    transposes."""

    import torch

    import radeon_kernels as rk

    m, n, k = 256, 384, 512
    gen = torch.Generator().manual_seed(11)
    a = seeded((m, k), 0, "uniform", dtype, gen)
    b = seeded((k, n), 0, "uniform", dtype, gen)
    g = seeded((m, n), 0, "uniform", dtype, gen)
    a_dev = a.cuda().requires_grad_(True)
    b_dev = b.cuda().requires_grad_(True)
    c = rk.gemm(a_dev, b_dev)
    c.backward(g.cuda())
    ga_bits, ga32 = oracle.gemm(to_bits(g), to_bits(b.t().contiguous()), dtype)
    gb_bits, gb32 = oracle.gemm(to_bits(a.t().contiguous()), to_bits(g), dtype)
    oracle.assert_parity(to_bits(a_dev.grad), ga_bits, ga32, dtype)
    oracle.assert_parity(to_bits(b_dev.grad), gb_bits, gb32, dtype)


def test_gemv_backward_and_transposed_weight():
    """gemv's weight gradient (grad^T @ x, "tn") and a weight given as the transpose of a
    dense [K, N] matrix (run as the nn GEMM x @ stored)."""

    import torch

    import radeon_kernels as rk

    m, n, k = 16, 1024, 512
    gen = torch.Generator().manual_seed(12)
    x = seeded((m, k), 0, "uniform", "bf16", gen)
    w = seeded((n, k), 0, "uniform", "bf16", gen)
    g = seeded((m, n), 0, "uniform", "bf16", gen)
    x_dev = x.cuda().requires_grad_(True)
    w_dev = w.cuda().requires_grad_(True)
    out = rk.gemv(x_dev, w_dev)
    out.backward(g.cuda())
    gx_bits, gx32 = oracle.gemm(to_bits(g), to_bits(w), "bf16")
    gw_bits, gw32 = oracle.gemm(to_bits(g.t().contiguous()), to_bits(x), "bf16")
    oracle.assert_parity(to_bits(x_dev.grad), gx_bits, gx32, "bf16")
    oracle.assert_parity(to_bits(w_dev.grad), gw_bits, gw32, "bf16")

    w_view = w.t().contiguous().cuda().t()  # [N, K] view of a dense [K, N] matrix
    out2 = rk.gemv(x.cuda(), w_view)
    o_bits, o32 = oracle.gemm(to_bits(x), to_bits(w.t().contiguous()), "bf16")
    oracle.assert_parity(to_bits(out2), o_bits, o32, "bf16")


def test_fresh_thread_encodes_tensor_maps():
    """A thread that never set its device (as PyTorch's autograd workers) calls the library
    first: the tensor-map encode must find a current context.  Shapes no other test uses, so
    no cached map hides the encode."""

    import threading

    import torch

    a, b, a_stored, b_stored = _operands("nt", 72, 136, 104, "bf16")
    a_dev, b_dev = a_stored.cuda(), b_stored.cuda()
    c = torch.empty(72, 136, dtype=torch.bfloat16, device="cuda")
    torch.cuda.synchronize()
    result = {}

    lib = _native.library()
    ptrs = [ctypes.c_void_p(t.data_ptr()) for t in (a_dev, b_dev, c)]

    def run():  # no torch call on this thread: the library is its first CUDA user
        result["status"] = lib.rk_gemm_layout(*ptrs, 72, 136, 104, 1, 1, GEMM["tc_1sm"], None)
        result["error"] = lib.rk_last_error()

    worker = threading.Thread(target=run)
    worker.start()
    worker.join()
    assert result["status"] == _native.RK_OK, result
    torch.cuda.synchronize()
    c_bits, c32 = oracle.gemm(to_bits(a), to_bits(b), "bf16")
    oracle.assert_parity(to_bits(c), c_bits, c32, "bf16")

