"""Backward kernels of silu_mul, rms_norm, add_rms_norm (and the fused gemm_swiglu's
autograd path) against the oracle and the reference's own autograd fixtures.

The reference runs inputs that require gradients through its torch fallbacks, so its
gradients are the autograd of those fp32 graphs (tests/golden/grad_*.npz hold them); the
oracle restates the same chain rule and is pinned to those fixtures on the CPU.  Gate:
oracle.assert_gradient (NaN where the reference has NaN; one representable step, or within
2^-14 of the terms' magnitude where terms cancel or long fp32 sums differ in order).
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import golden_cases
from gpu_util import DTYPE_CODE, device_status, seeded, stream_handle, to_bits, to_device
from oracle import oracle
from radeon_kernels import _native

pytestmark = pytest.mark.gpu


def _load(path):
    data = np.load(path)
    return {key: data[key] for key in data.files}


def _check_norm(got_x, got_w, ref, dt, ref_x_bits=None, ref_w_bits=None):
    """Kernel gradients against the oracle (bits + fp32 + scales), and, when given, against
    the reference's own rounded gradients with the oracle's fp32 values and scales."""

    inter = ref.get("grad_x_intermediate")
    oracle.assert_gradient(to_bits(got_x), ref["grad_x"], ref["grad_x_fp32"], ref["grad_x_scale"], dt, intermediate=inter)
    if got_w is not None:
        oracle.assert_gradient(
            to_bits(got_w), ref["grad_weight"], ref["grad_weight_fp32"], ref["grad_weight_scale"], dt
        )
    if ref_x_bits is not None:
        oracle.assert_gradient(
            to_bits(got_x), ref_x_bits, ref["grad_x_fp32"], ref["grad_x_scale"], dt, intermediate=inter
        )
    if ref_w_bits is not None and got_w is not None:
        oracle.assert_gradient(
            to_bits(got_w), ref_w_bits, ref["grad_weight_fp32"], ref["grad_weight_scale"], dt
        )


# ------------------------------------------------------- the reference's fixtures
@pytest.mark.parametrize("path", golden_cases("grad_silu"), ids=lambda p: p.stem)
def test_silu_mul_backward_matches_reference_autograd(path):
    case = _load(path)
    dt = str(case["dtype"])
    ext = _native.extension()
    dg, du = ext.silu_mul_backward(to_device(case["dy"], dt), to_device(case["gate"], dt), to_device(case["up"], dt))
    ref = oracle.silu_mul_backward(case["dy"], case["gate"], case["up"], dt)
    for key, got in (("grad_gate", dg), ("grad_up", du)):
        oracle.assert_gradient(to_bits(got), case[f"{key}_ref"], ref[f"{key}_fp32"], ref[f"{key}_scale"], dt)
        oracle.assert_gradient(to_bits(got), ref[key], ref[f"{key}_fp32"], ref[f"{key}_scale"], dt)


@pytest.mark.parametrize("path", golden_cases("grad_rms"), ids=lambda p: p.stem)
def test_rms_norm_backward_matches_reference_autograd(path):
    case = _load(path)
    dt, eps = str(case["dtype"]), float(case["eps"])
    ext = _native.extension()
    dx, dw = ext.rms_norm_backward(
        to_device(case["dy"], dt), to_device(case["x"], dt), to_device(case["weight"], dt), eps, True
    )
    ref = oracle.rms_norm_backward(case["dy"], case["x"], case["weight"], eps, dt)
    _check_norm(dx, dw, ref, dt, case["grad_x_ref"], case["grad_weight_ref"])


@pytest.mark.parametrize("path", golden_cases("grad_add_rms"), ids=lambda p: p.stem)
def test_add_rms_norm_backward_matches_reference_autograd(path):
    case = _load(path)
    dt, eps = str(case["dtype"]), float(case["eps"])
    dres = case.get("dres")
    ext = _native.extension()
    dx, dr, dw = ext.add_rms_norm_backward(
        to_device(case["dy"], dt),
        None if dres is None else to_device(dres, dt),
        to_device(case["residual_out"], dt),
        to_device(case["weight"], dt),
        eps,
        True,
    )
    assert np.array_equal(to_bits(dx), to_bits(dr))
    ref = oracle.add_rms_norm_backward(case["dy"], dres, case["residual_out"], case["weight"], eps, dt)
    _check_norm(dx, dw, ref, dt, case["grad_x_ref"], case["grad_weight_ref"])


# ------------------------------------------------------------- workload sizes
# The reference's workloads (benchmarks/workloads/rms_norm-1.0.yaml:11-14,
# add_rms_norm-1.0.yaml, swiglu-1.0.yaml:12-15).
NORM_SHAPES = [(1, 4096), (128, 4096), (2048, 4096), (1024, 8192), (7, 20000), (300, 13)]
SILU_SHAPES = [(1, 11008), (128, 11008), (1024, 11008), (512, 28672), (5, 13)]


@pytest.mark.parametrize("dt", ["bf16", "fp16"])
@pytest.mark.parametrize("shape", SILU_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_silu_mul_backward_workloads(shape, dt):
    gen = __import__("torch").Generator().manual_seed(shape[0] * 7 + shape[1])
    dy, g, u = (seeded(shape, 0, "normal", dt, gen) for _ in range(3))
    dg, du = _native.extension().silu_mul_backward(dy.cuda(), g.cuda(), u.cuda())
    ref = oracle.silu_mul_backward(to_bits(dy), to_bits(g), to_bits(u), dt)
    oracle.assert_gradient(to_bits(dg), ref["grad_gate"], ref["grad_gate_fp32"], ref["grad_gate_scale"], dt)
    oracle.assert_gradient(to_bits(du), ref["grad_up"], ref["grad_up_fp32"], ref["grad_up_scale"], dt)


@pytest.mark.parametrize("dt", ["bf16", "fp16"])
@pytest.mark.parametrize("shape", NORM_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_norm_backward_workloads(shape, dt):
    import torch

    tokens, hidden = shape
    gen = torch.Generator().manual_seed(tokens * 3 + hidden)
    dy, x, dres = (seeded(shape, 0, "normal", dt, gen) for _ in range(3))
    w = (1 + 0.1 * torch.randn((hidden,), generator=gen)).to(dy.dtype)
    ext = _native.extension()
    dx, dw = ext.rms_norm_backward(dy.cuda(), x.cuda(), w.cuda(), 1e-6, True)
    ref = oracle.rms_norm_backward(to_bits(dy), to_bits(x), to_bits(w), 1e-6, dt)
    _check_norm(dx, dw, ref, dt)
    # add_rms_norm with and without a residual_out gradient (x plays residual_out)
    for with_dres in (True, False):
        dx, dr, dw = ext.add_rms_norm_backward(
            dy.cuda(), dres.cuda() if with_dres else None, x.cuda(), w.cuda(), 1e-6, True
        )
        ref = oracle.add_rms_norm_backward(to_bits(dy), to_bits(dres) if with_dres else None, to_bits(x), to_bits(w), 1e-6, dt)
        _check_norm(dx, dw, ref, dt)
        assert np.array_equal(to_bits(dx), to_bits(dr))
    torch.cuda.synchronize()
    assert device_status() == _native.RK_OK


def test_weight_gradient_is_deterministic_and_optional():
    import torch

    gen = torch.Generator().manual_seed(9)
    dy, x = (seeded((2048, 4096), 0, "normal", "bf16", gen).cuda() for _ in range(2))
    w = torch.ones(4096, dtype=torch.bfloat16, device="cuda")
    ext = _native.extension()
    runs = [ext.rms_norm_backward(dy, x, w, 1e-6, True) for _ in range(3)]
    for dx, dw in runs[1:]:
        assert torch.equal(dx.view(torch.int16), runs[0][0].view(torch.int16))
        assert torch.equal(dw.view(torch.int16), runs[0][1].view(torch.int16))
    dx_only, none = ext.rms_norm_backward(dy, x, w, 1e-6, False)
    assert none is None
    assert torch.equal(dx_only.view(torch.int16), runs[0][0].view(torch.int16))


def test_edges_through_the_c_abi():
    """tokens == 0 zero-fills the weight gradient; hidden beyond the shared-memory
    accumulators is refused with a weight gradient and runs without one; a workspace
    smaller than the query's answer is refused."""

    import torch

    lib = _native.library()
    s = stream_handle()
    w = torch.ones(64, dtype=torch.float16, device="cuda")
    dw = torch.full((64,), 3.0, dtype=torch.float16, device="cuda")
    empty = torch.empty(0, 64, dtype=torch.float16, device="cuda")
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    assert lib.rk_rms_norm_backward(p(empty), p(empty), p(w), p(empty), p(dw), 0, 64, 1e-6,
                                    DTYPE_CODE["fp16"], None, 0, s) == _native.RK_OK
    torch.cuda.synchronize()
    assert torch.count_nonzero(dw).item() == 0

    big = 65536
    x = torch.randn(2, big, device="cuda").to(torch.float16)
    wb = torch.ones(big, dtype=torch.float16, device="cuda")
    dx = torch.empty_like(x)
    dwb = torch.empty_like(wb)
    size = ctypes.c_size_t(0)
    assert lib.rk_rms_norm_backward_workspace_size(2, big, ctypes.byref(size)) == _native.RK_OK
    ws = torch.empty(size.value, dtype=torch.uint8, device="cuda")
    assert lib.rk_rms_norm_backward(p(x), p(x), p(wb), p(dx), p(dwb), 2, big, 1e-6, DTYPE_CODE["fp16"],
                                    p(ws), size.value, s) == _native.RK_ERR_UNSUPPORTED
    assert lib.rk_rms_norm_backward(p(x), p(x), p(wb), p(dx), None, 2, big, 1e-6, DTYPE_CODE["fp16"],
                                    None, 0, s) == _native.RK_OK
    torch.cuda.synchronize()
    ref = oracle.rms_norm_backward(to_bits(x), to_bits(x), to_bits(wb), 1e-6, "fp16")
    oracle.assert_gradient(to_bits(dx), ref["grad_x"], ref["grad_x_fp32"], ref["grad_x_scale"], "fp16")

    x = torch.randn(300, 4096, device="cuda").to(torch.float16)
    w = torch.ones(4096, dtype=torch.float16, device="cuda")
    assert lib.rk_rms_norm_backward_workspace_size(300, 4096, ctypes.byref(size)) == _native.RK_OK
    ws = torch.empty(size.value, dtype=torch.uint8, device="cuda")
    dx, dw = torch.empty_like(x), torch.empty_like(w)
    assert lib.rk_rms_norm_backward(p(x), p(x), p(w), p(dx), p(dw), 300, 4096, 1e-6, DTYPE_CODE["fp16"],
                                    p(ws), size.value - 16, s) == _native.RK_ERR_INVALID_ARGUMENT
    assert lib.rk_rms_norm_backward(p(x), p(x), p(w), p(dx), p(dw), 300, 4096, 1e-6, DTYPE_CODE["fp16"],
                                    p(ws), size.value, s) == _native.RK_OK
    torch.cuda.synchronize()
    ref = oracle.rms_norm_backward(to_bits(x), to_bits(x), to_bits(w), 1e-6, "fp16")
    _check_norm(dx, dw, ref, "fp16")


# ----------------------------------------------------------------- public API
def test_public_api_autograd():
    """rk.silu_mul / rk.rms_norm / rk.add_rms_norm with inputs that require gradients: the
    cuda provider's autograd nodes run the backward kernels; gradients match the oracle."""

    import torch

    import radeon_kernels as rk

    gen = torch.Generator().manual_seed(21)
    t, h = 64, 1024
    g, u, dy, x, r, dres = (seeded((t, h), 0, "normal", "bf16", gen) for _ in range(6))
    w = (1 + 0.1 * torch.randn((h,), generator=gen)).to(torch.bfloat16)

    gd, ud = g.cuda().requires_grad_(True), u.cuda().requires_grad_(True)
    rk.silu_mul(gd, ud).backward(dy.cuda())
    ref = oracle.silu_mul_backward(to_bits(dy), to_bits(g), to_bits(u), "bf16")
    oracle.assert_gradient(to_bits(gd.grad), ref["grad_gate"], ref["grad_gate_fp32"], ref["grad_gate_scale"], "bf16")
    oracle.assert_gradient(to_bits(ud.grad), ref["grad_up"], ref["grad_up_fp32"], ref["grad_up_scale"], "bf16")

    xd, wd = x.cuda().requires_grad_(True), w.cuda().requires_grad_(True)
    rk.rms_norm(xd, wd).backward(dy.cuda())
    ref = oracle.rms_norm_backward(to_bits(dy), to_bits(x), to_bits(w), 1e-6, "bf16")
    _check_norm(xd.grad, wd.grad, ref, "bf16")

    for both in (True, False):
        xd, rd, wd = (t_.cuda().requires_grad_(True) for t_ in (x, r, w))
        out, res_out = rk.add_rms_norm(xd, rd, wd)
        if both:
            torch.autograd.backward([out, res_out], [dy.cuda(), dres.cuda()])
        else:
            out.backward(dy.cuda())
        ref = oracle.add_rms_norm_backward(
            to_bits(dy), to_bits(dres) if both else None, to_bits(res_out), to_bits(w), 1e-6, "bf16"
        )
        _check_norm(xd.grad, wd.grad, ref, "bf16")
        assert np.array_equal(to_bits(xd.grad), to_bits(rd.grad))


def test_gemm_swiglu_backward_is_the_composition_gradient():
    """rk.gemm_swiglu's gradients equal those of rk.gemm -> rk.silu_mul (the composition it
    replaces): the oracle's GEMM, silu_mul backward and the two GEMM gradients, GEMM gate."""

    import torch

    import radeon_kernels as rk

    m, n, k = 256, 256, 512
    gen = torch.Generator().manual_seed(22)
    a = seeded((m, k), 0, "normal/512", "bf16", gen)
    b = seeded((k, 2 * n), 0, "normal", "bf16", gen)
    dy = seeded((m, n), 0, "normal", "bf16", gen)
    ad, bd = a.cuda().requires_grad_(True), b.cuda().requires_grad_(True)
    rk.gemm_swiglu(ad, bd).backward(dy.cuda())

    # The same steps through the binding (deterministic kernels: the autograd path must
    # give identical bits), each step checked against the oracle on its own inputs.
    ext = _native.extension()
    y = ext.gemm(a.cuda(), b.cuda(), 0)
    y_bits, y32 = oracle.gemm(to_bits(a), to_bits(b), "bf16")
    oracle.assert_parity(to_bits(y), y_bits, y32, "bf16")
    dg, du = ext.silu_mul_backward(dy.cuda(), y[:, :n].contiguous(), y[:, n:].contiguous())
    yk = to_bits(y)
    ref = oracle.silu_mul_backward(to_bits(dy), yk[:, :n], yk[:, n:], "bf16")
    oracle.assert_gradient(to_bits(dg), ref["grad_gate"], ref["grad_gate_fp32"], ref["grad_gate_scale"], "bf16")
    oracle.assert_gradient(to_bits(du), ref["grad_up"], ref["grad_up_fp32"], ref["grad_up_scale"], "bf16")
    dyy = torch.cat([dg, du], dim=1)
    ga = ext.gemm_views(dyy, b.cuda().t(), None, 0)
    gb = ext.gemm_views(a.cuda().t(), dyy, None, 0)
    assert torch.equal(ga.view(torch.int16), ad.grad.view(torch.int16))
    assert torch.equal(gb.view(torch.int16), bd.grad.view(torch.int16))
    dyy_bits = to_bits(dyy)
    ga_bits, ga32 = oracle.gemm(dyy_bits, np.ascontiguousarray(to_bits(b).T), "bf16")
    gb_bits, gb32 = oracle.gemm(np.ascontiguousarray(to_bits(a).T), dyy_bits, "bf16")
    oracle.assert_parity(to_bits(ga), ga_bits, ga32, "bf16")
    oracle.assert_parity(to_bits(gb), gb_bits, gb32, "bf16")


def test_nt_layout_inside_autograd_repro():
    """The nt GEMM of C = A @ B's activation gradient (dC @ B^T, 256 x 512 x 384), called on
    the main thread through the binding and through the C ABI, before autograd calls it."""

    import torch

    from gpu_util import abi_gemm_layout

    gen = torch.Generator().manual_seed(11)
    b = seeded((512, 384), 0, "uniform", "bf16", gen).cuda()
    g = seeded((256, 384), 0, "uniform", "bf16", gen).cuda()
    c = torch.empty(256, 512, dtype=torch.bfloat16, device="cuda")
    status = abi_gemm_layout(g, b, c, "nt", 0, "bf16")
    assert status == _native.RK_OK, (_native.status_text(status), _native.library().rk_last_error())
    out = _native.extension().gemm_views(g, b.t(), None, 0)
    c_bits, c32 = oracle.gemm(to_bits(g), np.ascontiguousarray(to_bits(b).T), "bf16")
    oracle.assert_parity(to_bits(out), c_bits, c32, "bf16")
    oracle.assert_parity(to_bits(c), c_bits, c32, "bf16")
