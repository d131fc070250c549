"""silu_mul / rms_norm / add_rms_norm kernels on a B200, through the C ABI (and the public API).

Gate (oracle.assert_elementwise): NaN exactly where the reference has NaN, at most one
representable step from the reference everywhere else; residual_out bit-exact.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import golden_cases
from gpu_util import DTYPE_CODE, device_status, seeded, stream_handle, to_bits, to_device, torch_dtype
from oracle import oracle
from radeon_kernels import _native

pytestmark = pytest.mark.gpu
SENTINEL = 0x7E7E  # a NaN pattern in both dtypes; guards must keep it


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _guarded(torch, rows, cols, dtype, pad=4096, offset=0):
    buf = torch.full((rows * cols + 2 * pad + offset,), SENTINEL, dtype=torch.int16, device="cuda")
    view = buf.view(torch_dtype(dtype))[pad + offset : pad + offset + rows * cols].view(rows, cols)
    return buf, view


def _guards_intact(buf, rows, cols, pad=4096, offset=0):
    bits = to_bits(buf)
    return bool(np.all(bits[: pad + offset] == SENTINEL) and np.all(bits[pad + offset + rows * cols :] == SENTINEL))


def silu_abi(gate, up, out, dtype):
    t, h = gate.shape
    return _native.library().rk_silu_mul(_ptr(gate), _ptr(up), _ptr(out), t, h, DTYPE_CODE[dtype], stream_handle())


def rms_abi(x, w, out, eps, dtype):
    t, h = x.shape
    return _native.library().rk_rms_norm(_ptr(x), _ptr(w), _ptr(out), t, h, eps, DTYPE_CODE[dtype], stream_handle())


def add_rms_abi(x, r, w, out, res_out, eps, dtype):
    t, h = x.shape
    return _native.library().rk_add_rms_norm(
        _ptr(x), _ptr(r), _ptr(w), _ptr(out), _ptr(res_out), t, h, eps, DTYPE_CODE[dtype], stream_handle()
    )


def _load(path):
    data = np.load(path)
    case = {key: data[key] for key in data.files}
    case["dtype"] = str(case["dtype"])
    return case


@pytest.mark.parametrize("path", golden_cases("silu"), ids=lambda p: p.stem)
def test_silu_mul_matches_reference_fixtures(path):
    import torch

    case = _load(path)
    dt = case["dtype"]
    t, h = case["gate"].shape
    buf, out = _guarded(torch, t, h, dt)
    assert silu_abi(to_device(case["gate"], dt), to_device(case["up"], dt), out, dt) == _native.RK_OK
    torch.cuda.synchronize()
    assert _guards_intact(buf, t, h)
    oracle.assert_elementwise(to_bits(out), case["out_ref"], dt)


@pytest.mark.parametrize("path", golden_cases("rms"), ids=lambda p: p.stem)
def test_rms_norm_matches_reference_fixtures(path):
    import torch

    case = _load(path)
    dt = case["dtype"]
    t, h = case["x"].shape
    buf, out = _guarded(torch, t, h, dt)
    assert rms_abi(to_device(case["x"], dt), to_device(case["weight"], dt), out, float(case["eps"]), dt) == _native.RK_OK
    torch.cuda.synchronize()
    assert _guards_intact(buf, t, h)
    oracle.assert_elementwise(to_bits(out), case["out_ref"], dt)


@pytest.mark.parametrize("path", golden_cases("add_rms"), ids=lambda p: p.stem)
def test_add_rms_norm_matches_reference_fixtures(path):
    import torch

    case = _load(path)
    dt = case["dtype"]
    t, h = case["x"].shape
    buf, out = _guarded(torch, t, h, dt)
    rbuf, res_out = _guarded(torch, t, h, dt)
    x, r = to_device(case["x"], dt), to_device(case["residual"], dt)
    assert add_rms_abi(x, r, to_device(case["weight"], dt), out, res_out, float(case["eps"]), dt) == _native.RK_OK
    torch.cuda.synchronize()
    assert _guards_intact(buf, t, h) and _guards_intact(rbuf, t, h)
    assert np.array_equal(to_bits(res_out), case["residual_out_ref"])
    oracle.assert_elementwise(to_bits(out), case["out_ref"], dt)
    assert np.array_equal(to_bits(x), case["x"]) and np.array_equal(to_bits(r), case["residual"])  # inputs untouched


# The reference's workload cases (benchmarks/workloads/swiglu-1.0.yaml, add_rms_norm-1.0.yaml).
SILU_WORKLOADS = [(1, 11008), (128, 11008), (1024, 11008), (512, 28672)]
NORM_WORKLOADS = [(1, 4096), (128, 4096), (2048, 4096), (1024, 8192)]
# Prefill rows walked two (or three, past the resident capacity) per CTA, with a CTA left a
# single row: 1201 rows; 12000 rows of 1024.
NORM_WORKLOADS += [(1201, 2048), (12000, 1024)]


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("tokens, hidden", SILU_WORKLOADS)
def test_silu_mul_workloads(tokens, hidden, dtype):
    import torch

    gen = torch.Generator().manual_seed(tokens + hidden)
    gate = seeded((tokens, hidden), 0, "normal", dtype, gen)
    up = seeded((tokens, hidden), 0, "normal", dtype, gen)
    out = torch.empty(tokens, hidden, dtype=torch_dtype(dtype), device="cuda")
    assert silu_abi(gate.cuda(), up.cuda(), out, dtype) == _native.RK_OK
    again = torch.empty_like(out)
    assert silu_abi(gate.cuda(), up.cuda(), again, dtype) == _native.RK_OK
    torch.cuda.synchronize()
    ref, _ = oracle.silu_mul(to_bits(gate), to_bits(up), dtype)
    oracle.assert_elementwise(to_bits(out), ref, dtype)
    assert torch.equal(out.view(torch.int16), again.view(torch.int16))


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("tokens, hidden", NORM_WORKLOADS)
def test_add_rms_norm_workloads(tokens, hidden, dtype):
    import torch

    gen = torch.Generator().manual_seed(tokens * 7 + hidden)
    x = seeded((tokens, hidden), 0, "normal", dtype, gen)
    r = seeded((tokens, hidden), 0, "normal", dtype, gen)
    w = (1 + 0.1 * torch.randn((hidden,), generator=gen)).to(torch_dtype(dtype))
    out = torch.empty(tokens, hidden, dtype=torch_dtype(dtype), device="cuda")
    res_out = torch.empty_like(out)
    norm_only = torch.empty_like(out)
    assert add_rms_abi(x.cuda(), r.cuda(), w.cuda(), out, res_out, 1e-6, dtype) == _native.RK_OK
    assert rms_abi(x.cuda(), w.cuda(), norm_only, 1e-6, dtype) == _native.RK_OK
    torch.cuda.synchronize()
    ref, ref_res, _ = oracle.add_rms_norm(to_bits(x), to_bits(r), to_bits(w), 1e-6, dtype)
    assert np.array_equal(to_bits(res_out), ref_res)
    oracle.assert_elementwise(to_bits(out), ref, dtype)
    ref_norm, _ = oracle.rms_norm(to_bits(x), to_bits(w), 1e-6, dtype)
    oracle.assert_elementwise(to_bits(norm_only), ref_norm, dtype)


@pytest.mark.parametrize("offset", [0, 1])  # 1: every pointer 2 bytes off 16-byte alignment -> scalar path
@pytest.mark.parametrize(
    "tokens, hidden",
    # few rows: a CTA per row; >= 2 x SMs rows (aligned): a warp per row
    [(3, 4100), (2, 7), (5, 24), (1, 33000), (400, 16392), (300, 24), (1000, 4104)],
)
def test_ragged_and_unaligned_shapes(tokens, hidden, offset):
    import torch

    dtype = "bf16"
    gen = torch.Generator().manual_seed(hidden)

    def placed(t):
        buf = torch.empty(t.numel() + 8, dtype=t.dtype, device="cuda")
        view = buf[offset : offset + t.numel()].view(t.shape)
        view.copy_(t.cuda())
        return view

    x = placed(seeded((tokens, hidden), 0, "normal", dtype, gen))
    r = placed(seeded((tokens, hidden), 0, "normal", dtype, gen))
    w = placed((1 + 0.1 * torch.randn((hidden,), generator=gen)).to(torch.bfloat16))
    obuf, out = _guarded(torch, tokens, hidden, dtype, offset=offset)
    rbuf, res_out = _guarded(torch, tokens, hidden, dtype, offset=offset)
    sbuf, silu = _guarded(torch, tokens, hidden, dtype, offset=offset)
    assert add_rms_abi(x, r, w, out, res_out, 1e-5, dtype) == _native.RK_OK
    assert silu_abi(x, r, silu, dtype) == _native.RK_OK
    torch.cuda.synchronize()
    for buf in (obuf, rbuf, sbuf):
        assert _guards_intact(buf, tokens, hidden, offset=offset)
    ref, ref_res, _ = oracle.add_rms_norm(to_bits(x), to_bits(r), to_bits(w), 1e-5, dtype)
    assert np.array_equal(to_bits(res_out), ref_res)
    oracle.assert_elementwise(to_bits(out), ref, dtype)
    ref_silu, _ = oracle.silu_mul(to_bits(x), to_bits(r), dtype)
    oracle.assert_elementwise(to_bits(silu), ref_silu, dtype)


def test_empty_and_invalid_arguments():
    import torch

    lib = _native.library()
    x = torch.zeros(2, 8, dtype=torch.bfloat16, device="cuda")
    w = torch.ones(8, dtype=torch.bfloat16, device="cuda")
    bf16 = DTYPE_CODE["bf16"]
    assert lib.rk_silu_mul(None, None, None, 0, 8, bf16, stream_handle()) == _native.RK_OK
    assert lib.rk_rms_norm(_ptr(x), _ptr(w), _ptr(x), 0, 8, 1e-6, bf16, stream_handle()) == _native.RK_OK
    assert lib.rk_rms_norm(_ptr(x), _ptr(w), _ptr(x), 2, 8, 0.0, bf16, stream_handle()) == _native.RK_ERR_INVALID_ARGUMENT
    assert lib.rk_rms_norm(_ptr(x), _ptr(w), _ptr(x), 2, 8, float("nan"), bf16, stream_handle()) == _native.RK_ERR_INVALID_ARGUMENT
    assert lib.rk_rms_norm(_ptr(x), _ptr(w), _ptr(x), 2, 0, 1e-6, bf16, stream_handle()) == _native.RK_ERR_INVALID_ARGUMENT
    assert lib.rk_add_rms_norm(_ptr(x), None, _ptr(w), _ptr(x), _ptr(x), 2, 8, 1e-6, bf16, stream_handle()) == _native.RK_ERR_INVALID_ARGUMENT
    assert lib.rk_silu_mul(_ptr(x), _ptr(x), _ptr(x), 2, 8, 7, stream_handle()) == _native.RK_ERR_INVALID_ARGUMENT
    torch.cuda.synchronize()
    assert device_status() == _native.RK_OK


@pytest.fixture
def _fresh_runtimes():
    from radeon_kernels.ops._runtime import reset_operator_runtime

    reset_operator_runtime()
    yield


def test_public_api_dispatches_to_the_native_pack(_fresh_runtimes):
    import torch

    import radeon_kernels as rk

    gen = torch.Generator().manual_seed(5)
    x = seeded((16, 4096), 0, "normal", "fp16", gen).cuda()
    r = seeded((16, 4096), 0, "normal", "fp16", gen).cuda()
    w = (1 + 0.1 * torch.randn((4096,), generator=gen)).to(torch.float16).cuda()

    y = rk.silu_mul(x, r)
    record = rk.get_last_dispatch()
    assert record["operator"] == "swiglu" and record["selected"] == "native/silu_mul", record["reason"]
    oracle.assert_elementwise(to_bits(y), oracle.silu_mul(to_bits(x), to_bits(r), "fp16")[0], "fp16")

    y = rk.rms_norm(x, w, 1e-6)
    assert rk.get_last_dispatch()["selected"] == "native/rms_norm"
    oracle.assert_elementwise(to_bits(y), oracle.rms_norm(to_bits(x), to_bits(w), 1e-6, "fp16")[0], "fp16")

    y, s = rk.add_rms_norm(x, r, w)
    assert rk.get_last_dispatch()["selected"] == "native/add_rms_norm"
    ref, ref_res, _ = oracle.add_rms_norm(to_bits(x), to_bits(r), to_bits(w), 1e-6, "fp16")
    assert np.array_equal(to_bits(s), ref_res)
    oracle.assert_elementwise(to_bits(y), ref, "fp16")
    assert "selected: native/add_rms_norm" in rk.explain_last_dispatch()


def test_non_contiguous_and_grad_inputs_use_the_cuda_provider(_fresh_runtimes):
    import torch

    import radeon_kernels as rk

    gen = torch.Generator().manual_seed(6)
    base = seeded((64, 512), 0, "normal", "bf16", gen).cuda()
    gate = base[:, ::2]  # not contiguous
    up = seeded((64, 256), 0, "normal", "bf16", gen).cuda()
    y = rk.silu_mul(gate, up)
    assert rk.get_last_dispatch()["selected"] == "cuda/silu_mul"
    oracle.assert_elementwise(to_bits(y), oracle.silu_mul(to_bits(gate), to_bits(up), "bf16")[0], "bf16")

    w = torch.ones(256, dtype=torch.bfloat16, device="cuda", requires_grad=True)
    y = rk.rms_norm(up, w)
    assert rk.get_last_dispatch()["selected"] == "cuda/rms_norm"
    assert y.requires_grad
    oracle.assert_elementwise(to_bits(y), oracle.rms_norm(to_bits(up), to_bits(w), 1e-6, "bf16")[0], "bf16")
    y.float().sum().backward()  # the backward kernels (parity in test_gpu_backward.py)
    assert w.grad is not None and w.grad.shape == w.shape and torch.isfinite(w.grad.float()).all()
