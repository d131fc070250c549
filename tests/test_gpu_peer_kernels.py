"""The fused compute + all-gather kernels on one GPU.

``rk_gemv_allgather`` / ``rk_gemm_allgather`` normally run one rank per GPU (see
test_gpu_distributed.py).  Two single-GPU forms check them where only one GPU exists:

* a one-rank group: the kernels announce, store into the only output, count and advance the
  epoch exactly as with peers, and must reproduce the plain kernels (RK_GEMV_STREAM,
  RK_GEMM_TC_2SM) bit for bit, call after call;
* a two-rank group whose second rank is a local buffer that nobody drives: the wait for that
  rank's start flag can only run out.  With a 50 ms limit the kernel must give up, report
  RK_ERR_TIMEOUT through the status word, and leave the context usable.  No rank dies and
  no GPU faults: the flag is simply never set.
"""

from __future__ import annotations

import pytest

from gpu_util import seeded
from radeon_kernels import _native

pytestmark = pytest.mark.gpu

def _exchange(torch, m, n, dtype, ranks=1):
    """Per rank: one zeroed [control region | m x n] buffer laid out as
    radeon_kernels.distributed.peer does; returns (buffers, outputs, out_ptrs, ctl_ptrs)."""

    from radeon_kernels.distributed.peer import control_region_bytes

    ctl = control_region_bytes((m, n), ranks)
    esize = torch.empty((), dtype=dtype).element_size()
    bufs = [torch.zeros(ctl + m * n * esize, dtype=torch.uint8, device="cuda") for _ in range(ranks)]
    outs = [b[ctl:].view(dtype).view(m, n) for b in bufs]
    return bufs, outs, [o.data_ptr() for o in outs], [b.data_ptr() for b in bufs]


def _bits(t):
    import torch

    return t.contiguous().view(torch.int16)


@pytest.mark.parametrize("m", [1, 4, 32])
def test_one_rank_gemv_allgather_equals_the_stream_kernel(m):
    import torch

    ext = _native.extension()
    w = seeded((3000, 4096), 1, "normal/4096", "bf16").cuda()
    _, outs, out_ptrs, ctl_ptrs = _exchange(torch, m, 3000, torch.bfloat16)
    for call in range(3):  # epochs 1, 2, 3 on one control block
        x = seeded((m, 4096), 10 + call, "normal", "bf16").cuda()
        got = ext.gemv_allgather(x, w, outs[0], out_ptrs, ctl_ptrs, 0, 0).clone()
        want = ext.gemv_out(x, w, torch.empty(m, 3000, dtype=x.dtype, device="cuda"), _native.GEMV_VARIANTS["stream"])
        assert torch.equal(_bits(got), _bits(want)), call
    assert ext.device_status() == _native.RK_OK


@pytest.mark.parametrize("m, n, k", [(512, 8192, 1024), (16384 // 8, 57344 // 8, 8192)])
def test_one_rank_gemm_allgather_equals_the_pair_kernel(m, n, k):
    import torch

    ext = _native.extension()
    b = seeded((k, n), 2, "uniform16", "bf16").cuda()
    _, outs, out_ptrs, ctl_ptrs = _exchange(torch, m, n, torch.bfloat16)
    for call in range(2):
        a = seeded((m, k), 20 + call, "uniform16", "bf16").cuda()
        got = ext.gemm_allgather(a, b, outs[0], out_ptrs, ctl_ptrs, 0, 0).clone()
        want = ext.gemm_out(a, b, torch.empty(m, n, dtype=a.dtype, device="cuda"), _native.GEMM_VARIANTS["tc_2sm"])
        assert torch.equal(_bits(got), _bits(want)), call
    assert ext.device_status() == _native.RK_OK


@pytest.mark.parametrize("op", ["gemv", "gemm"])
def test_a_rank_that_never_starts_times_out_and_the_context_survives(op):
    import torch

    ext = _native.extension()
    m, n_block, k = (2, 1024, 1024) if op == "gemv" else (256, 1024, 512)
    _, outs, out_ptrs, ctl_ptrs = _exchange(torch, m, 2 * n_block, torch.bfloat16, ranks=2)
    limit_ns = 50_000_000
    if op == "gemv":
        x = seeded((m, k), 3, "normal", "bf16").cuda()
        w = seeded((n_block, k), 4, "normal/1024", "bf16").cuda()
        ext.gemv_allgather(x, w, outs[0], out_ptrs, ctl_ptrs, 0, limit_ns)
    else:
        a = seeded((m, k), 3, "uniform16", "bf16").cuda()
        b = seeded((k, n_block), 4, "uniform16", "bf16").cuda()
        ext.gemm_allgather(a, b, outs[0], out_ptrs, ctl_ptrs, 0, limit_ns)
    torch.cuda.synchronize()
    assert ext.device_status() == _native.RK_ERR_TIMEOUT
    assert ext.device_status() == _native.RK_OK  # read and cleared
    # The context is intact: an ordinary product still runs and is right.
    a = seeded((128, 256), 5, "uniform", "bf16").cuda()
    b = seeded((256, 128), 6, "uniform", "bf16").cuda()
    c = ext.gemm_out(a, b, torch.empty(128, 128, dtype=a.dtype, device="cuda"), 0)
    ref = (a.float() @ b.float()).to(torch.bfloat16)
    assert (c.float() - ref.float()).abs().max().item() <= 4e-3 * ref.float().abs().max().item()


def test_tail_half_tiles_match_whole_tiles():
    """[2048, 7168] is 224 tiles of 256 x 256 on 74 SM pairs: the last two run as four
    256 x 128 halves.  Each half of the matrix alone (112 tiles) runs whole tiles only; the
    products must agree bit for bit."""

    import torch

    ext = _native.extension()
    a = seeded((2048, 8192), 7, "uniform16", "bf16").cuda()
    b = seeded((8192, 7168), 8, "uniform16", "bf16").cuda()
    tc2 = _native.GEMM_VARIANTS["tc_2sm"]
    whole = ext.gemm_out(a, b, torch.empty(2048, 7168, dtype=a.dtype, device="cuda"), tc2)
    for lo in (0, 3584):
        part = ext.gemm_out(a, b[:, lo:lo + 3584].contiguous(), torch.empty(2048, 3584, dtype=a.dtype, device="cuda"), tc2)
        assert torch.equal(_bits(whole[:, lo:lo + 3584]), _bits(part))
