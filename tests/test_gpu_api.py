"""The public API on a B200: dispatch -> built-in sm_100a pack -> CUDA kernels."""

from __future__ import annotations

import pytest

from gpu_util import seeded, to_bits
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _fresh_runtimes():
    from radeon_kernels.ops._runtime import reset_operator_runtime
    from radeon_kernels.ops.gemm.api import reset_runtime

    reset_runtime()
    reset_operator_runtime()
    yield


def test_gemm_dispatches_to_the_native_pack_winner():
    import torch

    import radeon_kernels as rk

    a = seeded((1024, 1024), 0, "uniform", "bf16").cuda()
    b = seeded((1024, 1024), 1, "uniform", "bf16").cuda()
    c = rk.gemm(a, b)
    record = rk.get_last_dispatch()
    assert record["architecture"] == "sm_100a"
    assert record["selected"] == "native/gemm_out", record["reason"]
    assert record["entry_id"] == "gemm-sm100a-bf16-m1024-n1024-k1024"
    assert "loaded pack rk-sm100a" in record["reason"]
    ref_bits, ref32 = oracle.gemm(to_bits(a), to_bits(b), "bf16")
    oracle.assert_parity(to_bits(c), ref_bits, ref32, "bf16")
    out = torch.empty_like(c)
    assert rk.gemm(a, b, out=out) is out or rk.gemm(a, b, out=out).data_ptr() == out.data_ptr()
    assert torch.equal(out, c)
    assert "selected: native/gemm_out" in rk.explain_last_dispatch()


@pytest.mark.parametrize("m, entry", [(1, "m1-2"), (4, "m3-16"), (16, "m3-16")])
def test_gemv_dispatches_to_the_native_pack_winner(m, entry):
    """Config 3 through the public call: the stream kernel for M <= 2, tensor cores from M = 3."""

    import radeon_kernels as rk
    from radeon_kernels import _native

    x = seeded((m, 14336), 2, "normal", "fp16").cuda()
    w = seeded((4096, 14336), 2, "normal/14336", "fp16").cuda()
    out = rk.gemv(x, w)
    record = rk.get_last_dispatch()
    assert record["selected"] == "native/gemv", record["reason"]
    assert record["entry_id"] == f"gemv-sm100a-fp16-n4096-k14336-{entry}"
    from radeon_kernels.runtime.resources import builtin_dispatch_registry

    pinned = {e.id: e.launch.get("variant") for e in builtin_dispatch_registry().get("gemv", "1.0").entries
              if e.environment.architecture == "sm_100a"}
    assert pinned[record["entry_id"]] == _native.GEMV_VARIANTS["stream" if m <= 2 else "tc"]
    ref_bits, ref32 = oracle.gemv(to_bits(x), to_bits(w), "fp16")
    oracle.assert_parity(to_bits(out), ref_bits, ref32, "fp16")


def test_non_contiguous_inputs_run_the_cuda_fallback():
    import radeon_kernels as rk

    a = seeded((256, 192), 3, "uniform", "fp16").cuda()
    bt = seeded((128, 192), 4, "uniform", "fp16").cuda()
    b = bt.t()  # [192, 128], not contiguous
    c = rk.gemm(a, b)
    assert rk.get_last_dispatch()["selected"] == "cuda/gemm"
    ref_bits, ref32 = oracle.gemm(to_bits(a), to_bits(b.contiguous()), "fp16")
    oracle.assert_parity(to_bits(c), ref_bits, ref32, "fp16")


def test_autograd_runs_on_the_cuda_kernels():
    import torch

    import radeon_kernels as rk

    a = seeded((64, 96), 5, "uniform", "bf16").cuda().requires_grad_()
    b = seeded((96, 128), 6, "uniform", "bf16").cuda().requires_grad_()
    c = rk.gemm(a, b)
    assert rk.get_last_dispatch()["selected"] == "cuda/gemm"
    grad = seeded((64, 128), 7, "uniform", "bf16").cuda()
    c.backward(grad)
    ga = (grad.float() @ b.detach().float().t())
    gb = (a.detach().float().t() @ grad.float())
    assert (a.grad.float() - ga).abs().max().item() / ga.abs().max().item() <= 4e-3
    assert (b.grad.float() - gb).abs().max().item() / gb.abs().max().item() <= 4e-3
    x = seeded((2, 96), 8, "normal", "bf16").cuda().requires_grad_()
    w = seeded((40, 96), 9, "normal/96", "bf16").cuda().requires_grad_()
    y = rk.gemv(x, w)
    assert rk.get_last_dispatch()["selected"] == "cuda/gemv"
    y.sum().backward()
    assert torch.allclose(x.grad.float(), w.detach().float().sum(0).expand(2, 96), rtol=2e-2, atol=2e-2)


def test_odd_shapes_take_the_generic_kernel_through_the_pack():
    import radeon_kernels as rk

    a = seeded((5, 7), 1, "uniform", "bf16").cuda()
    b = seeded((7, 3), 2, "uniform", "bf16").cuda()
    c = rk.gemm(a, b)
    assert rk.get_last_dispatch()["selected"] == "native/gemm_out"
    ref_bits, ref32 = oracle.gemm(to_bits(a), to_bits(b), "bf16")
    oracle.assert_parity(to_bits(c), ref_bits, ref32, "bf16")


def test_tampered_pack_falls_back_to_cuda(tmp_path):
    import shutil

    from radeon_kernels.ops.gemm.api import GemmRuntime
    from radeon_kernels.runtime.packs import BUILTIN_PACK_ROOT

    copy = tmp_path / "packs"
    shutil.copytree(BUILTIN_PACK_ROOT, copy)
    artifact = copy / "rk-sm100a" / "lib" / "gemm" / "rk_sm100a.so"
    data = bytearray(artifact.read_bytes())
    data[-1] ^= 0xFF
    artifact.unlink()
    artifact.write_bytes(bytes(data))
    runtime = GemmRuntime(pack_roots=(), builtin_pack_roots=(copy,))
    a = seeded((128, 64), 1, "uniform", "bf16").cuda()
    b = seeded((64, 256), 2, "uniform", "bf16").cuda()
    c = runtime.execute(a, b)
    import radeon_kernels as rk

    record = rk.get_last_dispatch()
    assert record["selected"] == "cuda/gemm"
    assert "SHA-256 mismatch" in record["reason"]
    ref_bits, ref32 = oracle.gemm(to_bits(a), to_bits(b), "bf16")
    oracle.assert_parity(to_bits(c), ref_bits, ref32, "bf16")
