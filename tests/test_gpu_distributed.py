"""N-column sharded GEMM/GEMV on 2 GPUs (one process per GPU, NCCL), through the public API.

Each rank computes its block with this library's kernels; the all-gather + column-block
permute must reproduce the single-GPU product bit for bit (every output element is
accumulated in the same order whatever the column tiling).
"""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    import datetime

    sys.path.insert(0, str(REPO / "radeon-kernels_b200"))
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import radeon_kernels as rk
        from radeon_kernels.distributed import ShardedGemm, ShardedGemv

        gen = torch.Generator(device="cuda").manual_seed(4)
        a = ((torch.rand(512, 1024, device="cuda", generator=gen) * 2 - 1) / 16).to(torch.bfloat16)
        b = ((torch.rand(1024, 2048, device="cuda", generator=gen) * 2 - 1) / 16).to(torch.bfloat16)
        full = rk.gemm(a, b)
        sharded = ShardedGemm(b)(a, gather=True)
        x = torch.randn(4, 1024, device="cuda", generator=gen).to(torch.bfloat16)
        w = (torch.randn(4096, 1024, device="cuda", generator=gen) / 32).to(torch.bfloat16)
        gv_full = rk.gemv(x, w)
        gv = ShardedGemv(w)(x, gather=True)
        torch.cuda.synchronize()
        results[rank] = {
            "gemm_equal": bool(torch.equal(full.view(torch.int16), sharded.view(torch.int16))),
            "gemv_equal": bool(torch.equal(gv_full.view(torch.int16), gv.view(torch.int16))),
        }
        dist.barrier()
    except Exception as error:
        results[rank] = {"error": repr(error)[:300]}
    finally:
        dist.destroy_process_group()


def test_sharded_products_match_single_gpu_on_two_gpus():
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert not p.is_alive()
    assert dict(results) == {0: {"gemm_equal": True, "gemv_equal": True}, 1: {"gemm_equal": True, "gemv_equal": True}}
