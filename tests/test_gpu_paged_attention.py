"""rk_paged_attention_decode / rk.paged_attention_decode on a B200 (the reference's paged decode
attention, ops/paged_attention), through both kernels: the tcgen05 kernel (head_dim 64/128,
groups up to 16, block sizes 8-128) and the CUDA-core kernel (every case).  Gate:
oracle.assert_attention (NaN exactly where the reference has NaN, the GEMM parity rule
elsewhere; the tensor-core kernel rounds fp16 probabilities before the P.V product, so for
it fp16 gets the relative-to-max part of the gate)."""

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


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


PATH = {"tc": 2, "cuda": 1}


@pytest.fixture(params=["tc", "cuda"])
def kernel(request):
    """Pins rk_paged_attention_decode to one kernel for the test."""

    lib = _native.library()
    lib.rk_paged_attention_set_path(PATH[request.param])
    yield request.param
    lib.rk_paged_attention_set_path(0)


def _tc_takes(d, group, bs):
    return d in (64, 128) and group <= 16 and bs in (8, 16, 32, 64, 128)


def _gate(kernel, out, ref, ref32, dtype):
    oracle.assert_attention(to_bits(out), ref, ref32, dtype, rounded_p=kernel == "tc" and dtype == "fp16")


def run_abi(q, k, v, tables, lens, scale, dtype, out=None):
    import torch

    lib = _native.library()
    batch, hq, d = q.shape
    nb, bs, hkv, _ = k.shape
    maxb = tables.shape[1]
    need = ctypes.c_size_t(0)
    assert lib.rk_paged_attention_workspace_size(batch, hq, hkv, d, bs, maxb, ctypes.byref(need)) == _native.RK_OK
    ws = torch.empty(max(need.value, 1), dtype=torch.uint8, device="cuda")
    out = torch.empty_like(q) if out is None else out
    bits = 32 if tables.dtype == torch.int32 else 64
    st = lib.rk_paged_attention_decode(
        _ptr(q), _ptr(k), _ptr(v), _ptr(tables), _ptr(lens), _ptr(out), batch, hq, hkv, d, nb, bs, maxb,
        scale, DTYPE_CODE[dtype], bits, _ptr(ws), need.value, stream_handle(),
    )
    return st, out, need.value


def _load(path):
    data = np.load(path)
    return {key: data[key] for key in data.files}


@pytest.mark.parametrize("path", golden_cases("paged"), ids=lambda p: p.stem)
def test_matches_reference_fixtures(path, kernel):
    import torch

    case = _load(path)
    dt = str(case["dtype"])
    q, k, v = (to_device(case[n], dt) for n in ("q", "k", "v"))
    tables = torch.from_numpy(case["block_tables"]).cuda()
    lens = torch.from_numpy(case["context_lengths"]).cuda()
    st, out, _ = run_abi(q, k, v, tables, lens, float(case["scale"]), dt)
    if kernel == "tc" and not _tc_takes(q.shape[2], q.shape[1] // k.shape[2], k.shape[1]):
        assert st == _native.RK_ERR_UNSUPPORTED
        return
    assert st == _native.RK_OK
    torch.cuda.synchronize()
    assert device_status() == _native.RK_OK
    ref, ref32 = oracle.paged_attention_decode(
        case["q"], case["k"], case["v"], case["block_tables"], case["context_lengths"], float(case["scale"]), dt
    )
    _gate(kernel, out, case["out_ref"], ref32, dt)
    _gate(kernel, out, ref, ref32, dt)


def _random_case(torch, batch, hq, hkv, ctx, d, bs, dtype, seed, spare_blocks=3):
    gen = torch.Generator().manual_seed(seed)
    maxb = -(-ctx // bs)
    nb = batch * maxb + spare_blocks
    q = torch.randn((batch, hq, d), generator=gen).to(torch_dtype(dtype))
    k = torch.randn((nb, bs, hkv, d), generator=gen).to(torch_dtype(dtype))
    v = torch.randn((nb, bs, hkv, d), generator=gen).to(torch_dtype(dtype))
    perm = torch.randperm(nb, generator=gen)[: batch * maxb].view(batch, maxb)
    lengths = torch.full((batch,), ctx)
    return q, k, v, perm, lengths


# The reference's workload cases (benchmarks/workloads/paged_attention_decode-1.0.yaml):
# batch, query heads, kv heads, context, head_dim, block size.
WORKLOADS = [
    (1, 32, 8, 128, 128, 16),
    (1, 32, 8, 1024, 128, 16),
    (1, 32, 8, 4096, 128, 16),
    (8, 32, 8, 128, 128, 16),
    (8, 32, 8, 1024, 128, 16),
    (16, 32, 8, 2048, 128, 16),
    (4, 16, 16, 2048, 64, 32),
    (4, 32, 8, 1024, 256, 16),
]


@pytest.mark.parametrize("index", ["int32", "int64"])
@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("batch, hq, hkv, ctx, d, bs", WORKLOADS)
def test_reference_workloads(batch, hq, hkv, ctx, d, bs, dtype, index, kernel):
    import torch

    if index == "int64" and dtype == "fp16" and ctx < 2048:
        pytest.skip("index width is covered on the larger cases")
    if kernel == "tc" and not _tc_takes(d, hq // hkv, bs):
        pytest.skip("the tensor-core kernel does not take this shape (refusal checked on the fixtures)")
    q, k, v, tables, lens = _random_case(torch, batch, hq, hkv, ctx, d, bs, dtype, seed=batch * ctx + d)
    # ragged lengths inside the batch
    if batch > 1:
        lens = torch.tensor([max(1, ctx - 37 * i) for i in range(batch)])
    it = torch.int32 if index == "int32" else torch.int64
    tables_d, lens_d = tables.to(it).cuda(), lens.to(it).cuda()
    st, out, _ = run_abi(q.cuda(), k.cuda(), v.cuda(), tables_d, lens_d, 1.0 / math.sqrt(d), dtype)
    assert st == _native.RK_OK
    again = torch.empty_like(out)
    st2, again, _ = run_abi(q.cuda(), k.cuda(), v.cuda(), tables_d, lens_d, 1.0 / math.sqrt(d), dtype, out=again)
    torch.cuda.synchronize()
    assert st2 == _native.RK_OK and device_status() == _native.RK_OK
    assert torch.equal(out.view(torch.int16), again.view(torch.int16))
    ref, ref32 = oracle.paged_attention_decode(
        to_bits(q), to_bits(k), to_bits(v), tables.numpy(), lens.numpy(), 1.0 / math.sqrt(d), dtype
    )
    _gate(kernel, out, ref, ref32, dtype)


# Shapes at the tensor-core kernel's edges: 8- and 128-position blocks, MHA, a 16-head
# group, contexts ending inside a tile, many partitions (long context, one sequence), and
# groups of 2, 3, 6 and 8 heads (the kernel rounds a group up to 1, 4, 8 or 16 heads; with
# fewer than 16 query heads a Q box holds only the tensor's rows).
EDGES = [
    (2, 8, 8, 300, 128, 8),
    (2, 16, 1, 1000, 128, 128),
    (3, 4, 4, 129, 64, 64),
    (1, 32, 2, 8191, 128, 32),
    (5, 8, 2, 1, 64, 16),
    (2, 6, 2, 700, 128, 16),
    (3, 16, 2, 515, 64, 32),
    (2, 12, 2, 260, 128, 64),
    (2, 4, 2, 333, 128, 16),
]


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("batch, hq, hkv, ctx, d, bs", EDGES)
def test_tensor_core_edges(batch, hq, hkv, ctx, d, bs, dtype, kernel):
    import torch

    q, k, v, tables, lens = _random_case(torch, batch, hq, hkv, ctx, d, bs, dtype, seed=ctx + bs + hq)
    if batch > 1:
        lens = torch.tensor([max(1, ctx - 97 * i) for i in range(batch)])
    st, out, _ = run_abi(q.cuda(), k.cuda(), v.cuda(), tables.to(torch.int32).cuda(), lens.to(torch.int32).cuda(),
                         1.0 / math.sqrt(d), dtype)
    assert st == _native.RK_OK
    torch.cuda.synchronize()
    assert device_status() == _native.RK_OK
    ref, ref32 = oracle.paged_attention_decode(
        to_bits(q), to_bits(k), to_bits(v), tables.numpy(), lens.numpy(), 1.0 / math.sqrt(d), dtype
    )
    _gate(kernel, out, ref, ref32, dtype)


def test_many_items_per_cta_with_empty_sequences(kernel):
    """More (sequence, KV head) pairs than SMs, ragged lengths with empty sequences among
    them: the tensor-core kernel's CTAs walk several items each, some without tiles."""
    import torch

    batch, hq, hkv, d, bs, ctx = 300, 16, 2, 128, 16, 300
    q, k, v, tables, _ = _random_case(torch, batch, hq, hkv, ctx, d, bs, "bf16", seed=11)
    gen = torch.Generator().manual_seed(12)
    lens = torch.randint(0, ctx + 1, (batch,), generator=gen, dtype=torch.int32)
    lens[::7] = 0
    st, out, _ = run_abi(q.cuda(), k.cuda(), v.cuda(), tables.to(torch.int32).cuda(), lens.cuda(), 0.088, "bf16")
    assert st == _native.RK_OK
    torch.cuda.synchronize()
    assert device_status() == _native.RK_OK
    ref, ref32 = oracle.paged_attention_decode(
        to_bits(q), to_bits(k), to_bits(v), tables.numpy(), lens.numpy(), 0.088, "bf16"
    )
    live = (lens > 0).numpy()
    live_t = torch.from_numpy(live).to(out.device)
    _gate(kernel, out[live_t], ref[live], ref32[live], "bf16")
    assert bool(torch.isnan(out[~live_t].float()).all())


def test_lengths_zero_and_beyond_the_table_and_bad_block_indices(kernel):
    import torch

    q, k, v, tables, _ = _random_case(torch, 4, 8, 2, 96, 64, 16, "bf16", seed=5)
    # sequence 0: empty (NaN); 1: longer than its table (clamped); 2: normal; 3: one block
    # index out of range (skipped, reported)
    lens = torch.tensor([0, 10_000, 50, 96], dtype=torch.int32)
    bad = tables.clone().to(torch.int32)
    bad[3, 2] = k.shape[0] + 5
    st, out, _ = run_abi(q.cuda(), k.cuda(), v.cuda(), bad.cuda(), lens.cuda(), 0.125, "bf16")
    assert st == _native.RK_OK
    torch.cuda.synchronize()
    assert device_status() == _native.RK_ERR_INVALID_ARGUMENT  # the bad index was seen
    assert device_status() == _native.RK_OK  # and the word was cleared
    ref, ref32 = oracle.paged_attention_decode(
        to_bits(q[:3]), to_bits(k), to_bits(v), tables[:3].numpy(), np.array([0, 10_000, 50]), 0.125, "bf16"
    )
    _gate(kernel, out[:3], ref, ref32, "bf16")
    assert bool(torch.isnan(out[0].float()).all())
    assert bool(torch.isfinite(out[3].float()).all())


def test_public_api(monkeypatch):
    import torch

    import radeon_kernels as rk
    from radeon_kernels.ops._runtime import reset_operator_runtime

    reset_operator_runtime()
    q, k, v, tables, lens = _random_case(torch, 2, 32, 8, 300, 128, 16, "bf16", seed=7)
    args = (q.cuda(), k.cuda(), v.cuda(), tables.to(torch.int32).cuda(), lens.to(torch.int32).cuda())
    out = rk.paged_attention_decode(*args)
    record = rk.get_last_dispatch()
    assert record["operator"] == "paged_attention_decode"
    assert record["selected"] == "native/paged_attention_decode", record["reason"]
    ref, ref32 = oracle.paged_attention_decode(
        to_bits(q), to_bits(k), to_bits(v), tables.numpy(), lens.numpy(), 1.0 / math.sqrt(128), "bf16"
    )
    oracle.assert_attention(to_bits(out), ref, ref32, "bf16")
    out2 = rk.paged_attention_decode(*args, scale=0.05)
    ref2, ref32b = oracle.paged_attention_decode(
        to_bits(q), to_bits(k), to_bits(v), tables.numpy(), lens.numpy(), 0.05, "bf16"
    )
    oracle.assert_attention(to_bits(out2), ref2, ref32b, "bf16")
    with pytest.raises(ValueError, match="divisible"):
        rk.paged_attention_decode(args[0][:, :6], args[1], args[2], args[3], args[4])
    with pytest.raises(ValueError, match="inference-only"):
        rk.paged_attention_decode(args[0].clone().requires_grad_(), *args[1:])
