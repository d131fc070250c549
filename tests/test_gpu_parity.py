"""Parity of the CUDA kernels with the reference's arithmetic, through the C ABI.

Gate: max|C - C_ref| / max|C_ref| <= 4e-3 (bf16), 1e-3 (fp16),
C_ref = the fp32-accumulated product; plus at most one representable step from the
reference's own rounded output on every element not dominated by cancellation.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import golden_cases
from gpu_util import abi_gemm, abi_gemv, device_status, seeded, to_bits, to_device, torch_dtype
from oracle import oracle
from radeon_kernels import _native

pytestmark = pytest.mark.gpu
GEMM = _native.GEMM_VARIANTS
GEMV = _native.GEMV_VARIANTS
SENTINEL = 0x7E7E  # a NaN pattern in both fp16 and bf16


def _load(path):
    data = np.load(path)
    return {key: data[key] for key in data.files}


def _guarded(torch, rows, cols, dtype, pad=4096):
    """Output buffer inside a sentinel-filled guard region (bounds-check of the stores)."""

    buf = torch.full((rows * cols + 2 * pad,), SENTINEL, dtype=torch.int16, device="cuda").view(torch_dtype(dtype))
    return buf, buf[pad : pad + rows * cols].view(rows, cols)


def _guards_intact(buf, pad=4096):
    bits = to_bits(buf)
    return bool(np.all(bits[:pad] == SENTINEL) and np.all(bits[-pad:] == SENTINEL))


def _tc_ok(m, n, k):
    return n % 8 == 0 and k % 8 == 0 and k > 0 and m > 0


@pytest.mark.parametrize("variant", ["auto", "simt", "tc_1sm", "tc_2sm"])
@pytest.mark.parametrize("path", golden_cases("gemm"), ids=lambda p: p.stem)
def test_gemm_matches_reference_fixtures(path, variant):
    import torch

    case = _load(path)
    dtype = str(case["dtype"])
    a, b = to_device(case["a"], dtype), to_device(case["b"], dtype)
    m, k = a.shape
    n = b.shape[1]
    buf, c = _guarded(torch, m, n, dtype)
    a_before, b_before = to_bits(a), to_bits(b)
    status = abi_gemm(a, b, c, GEMM[variant], dtype)
    if variant in ("tc_1sm", "tc_2sm") and not _tc_ok(m, n, k) and m * n * k > 0:
        assert status == _native.RK_ERR_UNSUPPORTED
        return
    assert status == _native.RK_OK, _native.status_text(status)
    torch.cuda.synchronize()
    assert device_status() == _native.RK_OK
    assert _guards_intact(buf), "kernel wrote outside C"
    assert np.array_equal(to_bits(a), a_before) and np.array_equal(to_bits(b), b_before)
    oracle.assert_parity(to_bits(c), case["c_ref"], case["c_fp32"], dtype)


@pytest.mark.parametrize("variant", ["auto", "scalar", "stream", "tc"])
@pytest.mark.parametrize("path", golden_cases("gemv"), ids=lambda p: p.stem)
def test_gemv_matches_reference_fixtures(path, variant):
    import torch

    case = _load(path)
    dtype = str(case["dtype"])
    x, w = to_device(case["x"], dtype), to_device(case["w"], dtype)
    m, k = x.shape
    n = w.shape[0]
    buf, out = _guarded(torch, m, n, dtype)
    status = abi_gemv(x, w, out, GEMV[variant], dtype)
    if variant in ("stream", "tc") and k % 8 != 0:
        assert status == _native.RK_ERR_UNSUPPORTED
        return
    assert status == _native.RK_OK, _native.status_text(status)
    torch.cuda.synchronize()
    assert _guards_intact(buf)
    oracle.assert_parity(to_bits(out), case["out_reference"], case["out_fp32"], dtype)
    oracle.assert_parity(to_bits(out), case["out_fallback"], case["out_fp32"], dtype)


# ------------------------------------------------------------------ shape edges
EDGE_SHAPES = [
    (1, 8, 8),
    (1, 256, 64),
    (127, 248, 56),
    (129, 264, 72),
    (256, 256, 64),
    (300, 520, 1000),
    (64, 8, 4096),
    (1000, 1000, 8),
    (3, 17, 9),  # N, K not multiples of 8: generic kernel only
]


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("shape", EDGE_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_gemm_edge_shapes_against_oracle(shape, dtype):
    import torch

    m, n, k = shape
    gen = torch.Generator().manual_seed(m * 7 + n * 3 + k)
    a_cpu = seeded((m, k), 0, "uniform", dtype, gen)
    b_cpu = seeded((k, n), 0, "uniform", dtype, gen)
    c_bits, c32 = oracle.gemm(to_bits(a_cpu), to_bits(b_cpu), dtype)
    for variant in ("auto", "tc_1sm", "tc_2sm", "simt"):
        a, b = a_cpu.cuda(), b_cpu.cuda()
        buf, c = _guarded(torch, m, n, dtype)
        status = abi_gemm(a, b, c, GEMM[variant], dtype)
        if variant in ("tc_1sm", "tc_2sm") and not _tc_ok(m, n, k):
            assert status == _native.RK_ERR_UNSUPPORTED
            continue
        assert status == _native.RK_OK
        torch.cuda.synchronize()
        assert _guards_intact(buf)
        oracle.assert_parity(to_bits(c), c_bits, c32, dtype)


def test_unaligned_views_fall_back_to_the_generic_kernel():
    import torch

    base = seeded((1 + 64 * 128,), 0, "uniform", "bf16").cuda()
    a = base[1:].view(64, 128)  # 2-byte offset: not 16-byte aligned
    b = seeded((128, 64), 1, "uniform", "bf16").cuda()
    lib = _native.library()
    import ctypes

    assert lib.rk_gemm_select_variant(
        ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(b.data_ptr()), ctypes.c_void_p(0), 64, 64, 128, 1
    ) in (GEMM["simt"],)
    c = torch.empty(64, 64, dtype=torch.bfloat16, device="cuda")
    assert abi_gemm(a, b, c, GEMM["tc_1sm"], "bf16") == _native.RK_ERR_UNSUPPORTED
    assert abi_gemm(a, b, c, GEMM["auto"], "bf16") == _native.RK_OK
    c_bits, c32 = oracle.gemm(to_bits(a), to_bits(b), "bf16")
    oracle.assert_parity(to_bits(c), c_bits, c32, "bf16")


def test_empty_k_zero_fills():
    import torch

    a = torch.empty(5, 0, dtype=torch.float16, device="cuda")
    b = torch.empty(0, 9, dtype=torch.float16, device="cuda")
    c = torch.full((5, 9), 3.0, dtype=torch.float16, device="cuda")
    assert abi_gemm(a, b, c, 0, "fp16") == _native.RK_OK
    assert torch.count_nonzero(c).item() == 0


def test_non_finite_values_propagate():
    import torch

    a = seeded((128, 64), 0, "uniform", "bf16").cuda()
    b = seeded((64, 256), 1, "uniform", "bf16").cuda()
    a[3, 5] = float("inf")
    b[7, 9] = float("nan")
    for variant in ("tc_1sm", "simt"):
        c = torch.empty(128, 256, dtype=torch.bfloat16, device="cuda")
        assert abi_gemm(a, b, c, GEMM[variant], "bf16") == _native.RK_OK
        torch.cuda.synchronize()
        assert torch.isnan(c[:, 9]).all() and torch.isinf(c[3, :]).sum() + torch.isnan(c[3, :]).sum() == 256


# ------------------------------------------------------- BASELINE configurations
def _fp32_reference(a, b):
    import torch

    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return torch.mm(a.float(), b.float())
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def _check_full_gemm(a, b, dtype, rows, variant="auto"):
    """Full-size check against an fp32 product plus the C oracle on sampled rows."""

    import torch

    m, k = a.shape
    n = b.shape[1]
    c = torch.empty(m, n, dtype=a.dtype, device="cuda")
    assert abi_gemm(a, b, c, GEMM[variant], dtype) == _native.RK_OK
    torch.cuda.synchronize()
    assert device_status() == _native.RK_OK
    ref32 = _fp32_reference(a, b)
    scale = ref32.abs().max().item()
    err = (c.float() - ref32).abs().max().item() / scale
    assert err <= oracle.TOLERANCE[dtype], err
    b_bits = to_bits(b)
    a_rows = to_bits(a[rows])
    o_bits, o32 = oracle.gemm(a_rows, b_bits, dtype)
    oracle.assert_parity(to_bits(c[rows]), o_bits, o32, dtype)
    # determinism: a second launch is bit-identical
    c2 = torch.empty_like(c)
    assert abi_gemm(a, b, c2, GEMM[variant], dtype) == _native.RK_OK
    assert torch.equal(c.view(torch.int16), c2.view(torch.int16))
    return err


def test_config1_gemm_1024_bf16():
    gen = __import__("torch").Generator().manual_seed(0)
    a = seeded((1024, 1024), 0, "uniform", "bf16", gen).cuda()
    b = seeded((1024, 1024), 0, "uniform", "bf16", gen).cuda()
    _check_full_gemm(a, b, "bf16", [0, 1, 511, 1023])


@pytest.mark.parametrize("variant", ["auto", "tc_1sm", "tc_2sm"])
def test_config4_gemm_ffn_up_fp16(variant):
    gen = __import__("torch").Generator().manual_seed(3)
    a = seeded((4096, 4096), 3, "normal64", "fp16", gen).cuda()
    b = seeded((4096, 14336), 3, "normal64", "fp16", gen).cuda()
    _check_full_gemm(a, b, "fp16", [0, 4095], variant)


@pytest.fixture(scope="module")
def config5_inputs():
    """A then B drawn from one CPU torch.Generator seeded 4,
    uniform[-1, 1)/16, cast to bf16 (bitwise the inputs every rank of a sharded run draws)."""

    import torch

    gen = torch.Generator().manual_seed(4)
    a = seeded((16384, 8192), 4, "uniform16", "bf16", gen)
    b = seeded((8192, 57344), 4, "uniform16", "bf16", gen)
    return a, b


@pytest.mark.parametrize("shards", [1, 8])
def test_config5_gemm_large_bf16_column_blocks(shards, config5_inputs):
    import torch

    a_cpu, b_cpu = config5_inputs
    nb = 57344 // shards
    a = a_cpu.cuda()
    b = b_cpu[:, :nb].contiguous().cuda()  # rank 0's column block
    rows = [0, 16383] + sorted(np.random.default_rng(45).choice(16384, 6, replace=False).tolist())
    _check_full_gemm(a, b, "bf16", rows)
    del a, b
    torch.cuda.empty_cache()


@pytest.mark.parametrize("m", [1, 2, 4, 8, 16])
def test_config2_gemv_decode_bf16(m):
    import torch

    gen = torch.Generator().manual_seed(1)
    x = seeded((m, 8192), 1, "normal", "bf16", gen)
    w = seeded((8192, 8192), 1, "normal/8192", "bf16", gen)
    _check_full_gemv(x, w, "bf16")


@pytest.mark.parametrize("m", [1, 4, 8, 16])
def test_config3_gemv_ffn_down_fp16(m):
    import torch

    gen = torch.Generator().manual_seed(2)
    x = seeded((m, 14336), 2, "normal", "fp16", gen)
    w = seeded((4096, 14336), 2, "normal/14336", "fp16", gen)
    _check_full_gemv(x, w, "fp16")


def _check_full_gemv(x_cpu, w_cpu, dtype):
    import torch

    x, w = x_cpu.cuda(), w_cpu.cuda()
    out = torch.empty(x.shape[0], w.shape[0], dtype=x.dtype, device="cuda")
    assert abi_gemv(x, w, out, GEMV["auto"], dtype) == _native.RK_OK
    torch.cuda.synchronize()
    o_bits, o32 = oracle.gemv(to_bits(x_cpu), to_bits(w_cpu), dtype)
    oracle.assert_parity(to_bits(out), o_bits, o32, dtype)
    again = torch.empty_like(out)
    assert abi_gemv(x, w, again, GEMV["auto"], dtype) == _native.RK_OK
    assert torch.equal(out.view(torch.int16), again.view(torch.int16))


@pytest.mark.parametrize("rows, ks", [(1, 1), (2, 1), (4, 1), (2, 2), (2, 4), (1, 8), (4, 8)])
def test_gemv_tunings_agree(rows, ks):
    import torch

    gen = torch.Generator().manual_seed(9)
    x = seeded((3, 2048), 9, "normal", "bf16", gen)
    w = seeded((1000, 2048), 9, "normal/2048", "bf16", gen)
    o_bits, o32 = oracle.gemv(to_bits(x), to_bits(w), "bf16")
    lib = _native.library()
    lib.rk_gemv_set_tuning(rows, ks)
    try:
        out = torch.empty(3, 1000, dtype=torch.bfloat16, device="cuda")
        assert abi_gemv(x.cuda(), w.cuda(), out, GEMV["stream"], "bf16") == _native.RK_OK
        torch.cuda.synchronize()
    finally:
        lib.rk_gemv_set_tuning(0, 0)
    oracle.assert_parity(to_bits(out), o_bits, o32, "bf16")


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("m", [2, 3, 4, 5, 8, 16])
@pytest.mark.parametrize("n, k", [(1000, 2048), (37, 8200), (513, 4104), (64, 14336)])
def test_gemv_stream_skinny_m(m, n, k, dtype):
    """The CUDA-core stream kernel at M >= 2 (shared widening, packed FMAs, two pipeline
    stages up to M = 4): K slices of odd and ragged vector counts per lane, so the second
    stage runs past the slice end, against the oracle."""
    import torch

    gen = torch.Generator().manual_seed(100 + m)
    x = seeded((m, k), 100 + m, "normal", dtype, gen)
    w = seeded((n, k), 100 + m, f"normal/{k}", dtype, gen)
    o_bits, o32 = oracle.gemv(to_bits(x), to_bits(w), dtype)
    buf, out = _guarded(torch, m, n, dtype)
    assert abi_gemv(x.cuda(), w.cuda(), out, GEMV["stream"], dtype) == _native.RK_OK
    torch.cuda.synchronize()
    assert device_status() == _native.RK_OK
    assert _guards_intact(buf), "kernel wrote outside out"
    oracle.assert_parity(to_bits(out), o_bits, o32, dtype)


@pytest.mark.parametrize("cluster", [1, 2, 4, 8])
@pytest.mark.parametrize("m", [1, 5, 16, 17, 32])
def test_gemv_tensor_core_cluster_split_k(cluster, m):
    import torch

    gen = torch.Generator().manual_seed(11 + m)
    x = seeded((m, 4096 + 8), 11, "normal", "fp16", gen)  # K not a multiple of the 64-wide K block
    w = seeded((1000, 4096 + 8), 11, "normal/4104", "fp16", gen)  # N not a multiple of 128
    o_bits, o32 = oracle.gemv(to_bits(x), to_bits(w), "fp16")
    lib = _native.library()
    lib.rk_gemv_tc_set_cluster(cluster)
    try:
        buf, out = _guarded(torch, m, 1000, "fp16")
        assert abi_gemv(x.cuda(), w.cuda(), out, GEMV["tc"], "fp16") == _native.RK_OK
        torch.cuda.synchronize()
        assert device_status() == _native.RK_OK
    finally:
        lib.rk_gemv_tc_set_cluster(0)
    assert _guards_intact(buf)
    oracle.assert_parity(to_bits(out), o_bits, o32, "fp16")


@pytest.mark.parametrize("m", [1, 5, 16, 17, 32])
@pytest.mark.parametrize("n, k, cluster", [(1000, 4104, 2), (1000, 4104, 4), (4096, 14336, 0)])
def test_gemv_tensor_core_pushed_and_pulled_exchange_agree(m, n, k, cluster):
    """The cluster's partial sums reach the leader pulled (read through DSMEM) or pushed
    (stored into its receive area): the same additions in the same order, so the outputs
    agree bit for bit, and with the oracle.  cluster 0 is the automatic size (BASELINE
    config 3's weight, where the automatic exchange is the pushed one when every cluster
    of the grid fits at once)."""

    import torch

    gen = torch.Generator().manual_seed(17 + m + n)
    x = seeded((m, k), 17, "normal", "bf16", gen)
    w = seeded((n, k), 17, f"normal/{k}", "bf16", gen)
    o_bits, o32 = oracle.gemv(to_bits(x), to_bits(w), "bf16")
    lib = _native.library()
    lib.rk_debug_last_kernel.restype = ctypes.c_char_p
    outs, names = [], []
    lib.rk_gemv_tc_set_cluster(cluster)
    try:
        for exchange in (1, 2, 0):
            lib.rk_gemv_tc_set_exchange(exchange)
            buf, out = _guarded(torch, m, n, "bf16")
            assert abi_gemv(x.cuda(), w.cuda(), out, GEMV["tc"], "bf16") == _native.RK_OK
            names.append(lib.rk_debug_last_kernel().decode())
            torch.cuda.synchronize()
            assert device_status() == _native.RK_OK
            assert _guards_intact(buf)
            outs.append(out)
    finally:
        lib.rk_gemv_tc_set_exchange(0)
        lib.rk_gemv_tc_set_cluster(0)
    assert names[:2] == ["gemv_tc_kernel", "gemv_tc_kernel<push>"], names
    for other in outs[1:]:
        assert torch.equal(outs[0].view(torch.int16), other.view(torch.int16))
    oracle.assert_parity(to_bits(outs[1]), o_bits, o32, "bf16")


@pytest.mark.parametrize("m", [3, 5, 16, 17, 32])
@pytest.mark.parametrize("n, k", [(1000, 4104), (640, 14336), (8192, 8192)])
def test_gemv_tensor_core_workspace_split_k(m, n, k):
    """rk_gemv_ex: stream-K over independent CTAs meeting in a caller-owned workspace."""

    import ctypes

    import torch

    gen = torch.Generator().manual_seed(m + n)
    x = seeded((m, k), 13, "normal", "bf16", gen)
    w = seeded((n, k), 13, f"normal/{k}", "bf16", gen)
    o_bits, o32 = oracle.gemv(to_bits(x), to_bits(w), "bf16")
    lib = _native.library()
    need = ctypes.c_size_t(0)
    lib.rk_gemv_tc_set_cluster(-1)  # select stream-K (the workspace strategy)
    try:
        assert lib.rk_gemv_workspace_size(m, n, k, 1, GEMV["tc"], ctypes.byref(need)) == _native.RK_OK
        assert need.value > 0
        ws = torch.zeros(need.value + 4096, dtype=torch.uint8, device="cuda")
        outs = _run_stream_k(lib, x.cuda(), w.cuda(), ws, need.value, m, n, k)
    finally:
        lib.rk_gemv_tc_set_cluster(0)
    tiles = (n + 127) // 128
    assert int(ws[: 4 * tiles].view(torch.int32).abs().sum().item()) == 0  # tickets re-zeroed
    assert torch.equal(outs[0].view(torch.int16), outs[1].view(torch.int16))
    oracle.assert_parity(to_bits(outs[0]), o_bits, o32, "bf16")
    ws_default = ctypes.c_size_t(1)
    assert lib.rk_gemv_workspace_size(m, n, k, 1, GEMV["tc"], ctypes.byref(ws_default)) == _native.RK_OK
    assert ws_default.value == 0  # the default strategy needs no workspace


def _run_stream_k(lib, xd, wd, ws, need, m, n, k):
    import ctypes

    import torch

    outs = []
    for _ in range(2):  # the second call relies on the first leaving the tickets zeroed
        buf, out = _guarded(torch, m, n, "bf16")
        st = lib.rk_gemv_ex(
            ctypes.c_void_p(xd.data_ptr()), ctypes.c_void_p(wd.data_ptr()), ctypes.c_void_p(out.data_ptr()),
            m, n, k, 1, GEMV["tc"], ctypes.c_void_p(ws.data_ptr()), need,
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
        )
        assert st == _native.RK_OK, _native.status_text(st)
        torch.cuda.synchronize()
        assert _guards_intact(buf)
        outs.append(out.clone())
    assert device_status() == _native.RK_OK
    return outs


def test_gather_column_blocks_matches_permute():
    import ctypes

    import torch

    g, m, nb = 4, 33, 40
    blocks = torch.randn(g, m, nb, device="cuda").to(torch.bfloat16)
    out = torch.empty(m, g * nb, dtype=torch.bfloat16, device="cuda")
    st = _native.library().rk_gather_column_blocks(
        ctypes.c_void_p(blocks.data_ptr()), ctypes.c_void_p(out.data_ptr()), g, m, g * nb, 1,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
    )
    assert st == _native.RK_OK
    assert torch.equal(out, blocks.permute(1, 0, 2).reshape(m, g * nb))
    nb = 3  # scalar path
    blocks = torch.randn(g, m, nb, device="cuda").to(torch.float16)
    out = torch.empty(m, g * nb, dtype=torch.float16, device="cuda")
    st = _native.library().rk_gather_column_blocks(
        ctypes.c_void_p(blocks.data_ptr()), ctypes.c_void_p(out.data_ptr()), g, m, g * nb, 0,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
    )
    assert st == _native.RK_OK
    assert torch.equal(out, blocks.permute(1, 0, 2).reshape(m, g * nb))


@pytest.mark.parametrize(
    "op, variant, m, n, k",
    [
        ("gemv", "stream", 1, 4096, 4096),
        ("gemv", "tc", 16, 4096, 4096),
        ("gemm", "tc_1sm", 512, 1024, 1024),
        ("gemm", "tc_2sm", 512, 1024, 1024),
    ],
)
def test_programmatic_launch_is_result_neutral(op, variant, m, n, k):
    """Back-to-back launches with programmatic dependent launch on and off agree bit for bit.

    Each launch reads the previous launch's output directly as its input (a chain with
    N == K, no other kernel in between), so a kernel that touched global memory before its
    predecessor finished would read a stale operand.
    """

    import torch

    lib = _native.library()
    gen = torch.Generator().manual_seed(23)
    dtype = "bf16"
    chain = 4
    if op == "gemv":
        w_cpu = seeded((n, k), 23, f"normal/{k}", dtype, gen)
        x_cpu = seeded((m, k), 23, "normal", dtype, gen)
        w = w_cpu.cuda()
        results = {}
        for pdl in (0, 1):
            prev = lib.rk_set_programmatic_launch(pdl)
            try:
                xs = [x_cpu.cuda()]
                for _ in range(chain):
                    out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
                    assert abi_gemv(xs[-1], w, out, GEMV[variant], dtype) == _native.RK_OK
                    xs.append(out)
                torch.cuda.synchronize()
                assert device_status() == _native.RK_OK
            finally:
                lib.rk_set_programmatic_launch(prev)
            results[pdl] = [t.cpu() for t in xs[1:]]
        first_bits, first32 = oracle.gemv(to_bits(x_cpu), to_bits(w_cpu), dtype)
    else:
        a_cpu = seeded((m, k), 23, "normal", dtype, gen)
        b_cpu = seeded((k, n), 24, f"normal/{k}", dtype, gen)
        b = b_cpu.cuda()
        results = {}
        for pdl in (0, 1):
            prev = lib.rk_set_programmatic_launch(pdl)
            try:
                xs = [a_cpu.cuda()]
                for _ in range(chain):
                    c = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
                    assert abi_gemm(xs[-1], b, c, GEMM[variant], dtype) == _native.RK_OK
                    xs.append(c)
                torch.cuda.synchronize()
                assert device_status() == _native.RK_OK
            finally:
                lib.rk_set_programmatic_launch(prev)
            results[pdl] = [t.cpu() for t in xs[1:]]
        first_bits, first32 = oracle.gemm(to_bits(a_cpu), to_bits(b_cpu), dtype)
    for on, off in zip(results[1], results[0]):
        assert torch.equal(on.view(torch.int16), off.view(torch.int16))
    first = results[1][0]
    oracle.assert_parity(to_bits(first), first_bits, first32, dtype)
