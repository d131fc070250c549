"""rk.sdpa / rk_sdpa (tcgen05 flash attention) against the reference's own outputs and the
oracle (numpy restatement of ops/sdpa/reference.py:13-36).

Gate: oracle.assert_attention(..., rounded_p=True) -- NaN where the reference has NaN and
max|out - ref32| / max|ref32| <= 4e-3 (bf16) / 1e-3 (fp16); the probabilities are rounded to
the dtype before the P.V product on the tensor cores.
"""

from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest

from conftest import golden_cases
from gpu_util import DTYPE_CODE, device_status, stream_handle, to_bits, to_device, torch_dtype
from oracle import oracle
from radeon_kernels import _native

pytestmark = pytest.mark.gpu
SENTINEL = 0x7E7E


def _load(path):
    data = np.load(path)
    return {key: data[key] for key in data.files}


def _inputs(b, hq, hkv, s, d, dtype, seed, dist="uniform"):
    import torch

    gen = torch.Generator().manual_seed(seed)
    draw = (lambda shape: torch.rand(shape, generator=gen) * 0.25 - 0.125) if dist == "uniform" else (
        lambda shape: torch.randn(shape, generator=gen))
    tdt = torch_dtype(dtype)
    return draw((b, hq, s, d)).to(tdt), draw((b, hkv, s, d)).to(tdt), draw((b, hkv, s, d)).to(tdt)


def _abi_sdpa(q, k, v, out, causal, scale, dtype):
    lib = _native.library()
    b, hq, s, d = q.shape
    return lib.rk_sdpa(
        ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()), ctypes.c_void_p(v.data_ptr()),
        ctypes.c_void_p(out.data_ptr()), b, hq, k.shape[1], s, d, 1 if causal else 0, scale,
        DTYPE_CODE[dtype], stream_handle(),
    )


@pytest.mark.parametrize("path", golden_cases("sdpa"), ids=lambda p: p.stem)
def test_sdpa_matches_reference_fixtures(path):
    import radeon_kernels as rk

    case = _load(path)
    dt = str(case["dtype"])
    q, k, v = (to_device(case[n], dt) for n in ("q", "k", "v"))
    causal, scale = bool(case["is_causal"]), float(case["scale"])
    out = rk.sdpa(q, k, v, is_causal=causal, scale=scale)
    assert rk.get_last_dispatch()["selected"] == "native/sdpa"
    _, ref32 = oracle.sdpa(case["q"], case["k"], case["v"], causal, scale, dt)
    oracle.assert_attention(to_bits(out), case["out_ref"], ref32, dt, rounded_p=True)


# The reference's workloads (benchmarks/workloads/sdpa-1.0.yaml:12-19).
WORKLOADS = [
    (1, 16, 16, 128, 64, True),
    (1, 32, 8, 128, 128, True),
    (1, 32, 8, 256, 128, True),
    (1, 32, 8, 512, 128, True),
    (4, 32, 8, 128, 128, True),
    (8, 32, 8, 64, 128, True),
    (1, 16, 16, 256, 64, False),
    (2, 16, 4, 256, 256, True),
]


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("case", WORKLOADS, ids=lambda c: "b{}-h{}x{}-s{}-d{}-{}".format(*c[:5], "causal" if c[5] else "full"))
def test_sdpa_reference_workloads(case, dtype):
    import torch

    b, hq, hkv, s, d, causal = case
    q, k, v = _inputs(b, hq, hkv, s, d, dtype, seed=hq * 131 + s + d)
    scale = 1 / math.sqrt(d)
    buf = torch.full((q.numel() + 8192,), SENTINEL, dtype=torch.int16, device="cuda").view(q.dtype)
    out = buf[4096 : 4096 + q.numel()].view(q.shape)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    assert _abi_sdpa(qd, kd, vd, out, causal, scale, dtype) == _native.RK_OK
    torch.cuda.synchronize()
    assert device_status() == _native.RK_OK
    bits = to_bits(buf)
    assert np.all(bits[:4096] == SENTINEL) and np.all(bits[-4096:] == SENTINEL), "kernel wrote outside out"
    assert np.array_equal(to_bits(qd), to_bits(q)) and np.array_equal(to_bits(vd), to_bits(v))
    ref, ref32 = oracle.sdpa(to_bits(q), to_bits(k), to_bits(v), causal, scale, dtype)
    oracle.assert_attention(to_bits(out), ref, ref32, dtype, rounded_p=True)


@pytest.mark.parametrize(
    "shape",
    [(1, 2, 1, 1, 128, True), (1, 2, 2, 129, 64, True), (1, 4, 2, 1000, 128, True), (1, 4, 1, 1000, 128, False),
     (1, 2, 2, 2048, 128, True), (1, 2, 1, 700, 256, True), (2, 2, 2, 333, 256, False)],
    ids=lambda c: "b{}-h{}x{}-s{}-d{}-{}".format(*c[:5], "causal" if c[5] else "full"),
)
@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_sdpa_long_and_ragged_sequences(shape, dtype):
    """Many key tiles (online rescaling of O in TMEM), sequence ends inside a tile, one
    token, normal-distributed inputs (peaked softmax)."""

    b, hq, hkv, s, d, causal = shape
    q, k, v = _inputs(b, hq, hkv, s, d, dtype, seed=s * 7 + d, dist="normal")
    scale = 1 / math.sqrt(d)
    out = _native.extension().sdpa(q.cuda(), k.cuda(), v.cuda(), causal, scale)
    ref, ref32 = oracle.sdpa(to_bits(q), to_bits(k), to_bits(v), causal, scale, dtype)
    oracle.assert_attention(to_bits(out), ref, ref32, dtype, rounded_p=True)


@pytest.mark.parametrize("q_scale", [0.0, 1e-3, 3e-2])
@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_sdpa_near_uniform_attention(q_scale, dtype):
    """Scores near zero: every probability of a row is close to the same value, so a
    rounding of P that moves them all the same way must cancel in O / l (the row sum adds
    the probabilities as rounded for P V).  q_scale 0: exactly uniform attention."""

    b, hq, hkv, s, d = 1, 4, 2, 1500, 128
    q, k, v = _inputs(b, hq, hkv, s, d, dtype, seed=int(q_scale * 1e4) + 3, dist="normal")
    q = (q.float() * q_scale).to(q.dtype)
    scale = 1 / math.sqrt(d)
    for causal in (False, True):
        out = _native.extension().sdpa(q.cuda(), k.cuda(), v.cuda(), causal, scale)
        ref, ref32 = oracle.sdpa(to_bits(q), to_bits(k), to_bits(v), causal, scale, dtype)
        oracle.assert_attention(to_bits(out), ref, ref32, dtype, rounded_p=True)


def test_sdpa_is_deterministic_and_propagates_non_finite_values():
    import torch

    q, k, v = (t.cuda() for t in _inputs(1, 4, 2, 300, 128, "bf16", seed=5))
    ext = _native.extension()
    a = ext.sdpa(q, k, v, True, 0.1)
    b = ext.sdpa(q, k, v, True, 0.1)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    # A NaN key at position 200 is masked for queries before it (causal) and poisons the rows
    # from 200 on (their scores include it); a NaN query row only poisons itself.
    k2 = k.clone()
    k2[0, 0, 200, 5] = float("nan")
    q2 = q.clone()
    q2[0, 3, 50, 7] = float("nan")
    out = ext.sdpa(q2, k2, v, True, 0.1)
    ref, ref32 = oracle.sdpa(to_bits(q2), to_bits(k2), to_bits(v), True, 0.1, "bf16")
    oracle.assert_attention(to_bits(out), ref, ref32, "bf16", rounded_p=True)
    nan = torch.isnan(out.float())
    assert not nan[0, 0, :200].any() and nan[0, 0, 200:].all()
    assert nan[0, 3, 50].all() and not nan[0, 3, :50].any()


def test_sdpa_rejects_bad_arguments_through_the_c_abi():
    import torch

    lib = _native.library()
    q = torch.zeros(1, 4, 8, 64, dtype=torch.float16, device="cuda")
    k = torch.zeros(1, 3, 8, 64, dtype=torch.float16, device="cuda")
    out = torch.empty_like(q)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    s = stream_handle()
    assert lib.rk_sdpa(p(q), p(k), p(k), p(out), 1, 4, 3, 8, 64, 0, 0.1, 0, s) == _native.RK_ERR_INVALID_ARGUMENT
    assert lib.rk_sdpa(p(q), p(q), p(q), p(out), 1, 4, 4, 8, 96, 0, 0.1, 0, s) == _native.RK_ERR_INVALID_ARGUMENT
    assert lib.rk_sdpa(p(q), p(q), p(q), p(out), 1, 4, 4, 8, 64, 0, -1.0, 0, s) == _native.RK_ERR_INVALID_ARGUMENT
    assert lib.rk_sdpa(p(q), p(q), p(q), p(out), 1, 4, 4, 8, 64, 0, 0.1, 0, s) == _native.RK_OK
