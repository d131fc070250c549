"""N-column sharding plumbing on CPU gloo ranks (world size 2 and 3).

The per-rank products and the block permute are stood in for by torch on CPU here
(the product runs this library's CUDA kernels for both; those are covered by the
GPU tests).  What is tested: block bounds, that every rank computes exactly its block,
that the all-gather + permute layout reassembles the full row-major result, and that a
failing rank surfaces as an error on the others instead of a hang.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from radeon_kernels.distributed.shard import column_block


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _permute_cpu(blocks, out):
    # Reference of rk_gather_column_blocks: [G, M, N/G] -> [M, N].
    g, m, nb = blocks.shape
    out.copy_(blocks.permute(1, 0, 2).reshape(m, g * nb))
    return out


def _worker(rank, world, port, results, mode):
    import datetime

    import torch.distributed as dist

    from radeon_kernels.distributed.shard import ShardedGemm, ShardedGemv

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        if mode == "decide":
            results[rank] = _decide(rank, world)
            return
        gen = torch.Generator().manual_seed(0)
        a = torch.randn(5, 16, generator=gen)
        b = torch.randn(16, 6 * world, generator=gen)
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 fails before the collective")
        gemm = ShardedGemm(b, compute=lambda x, y: x @ y, permute=_permute_cpu)
        local = gemm(a)
        full = gemm(a, gather=True)
        x = torch.randn(3, 16, generator=gen)
        w = torch.randn(4 * world, 16, generator=gen)
        gemv = ShardedGemv(w, compute=lambda p, q: p @ q.t(), permute=_permute_cpu)
        results[rank] = {
            "block": (gemm.block.start, gemm.block.stop),
            "local_ok": bool(torch.allclose(local, (a @ b)[:, gemm.block.start : gemm.block.stop])),
            "full_ok": bool(torch.allclose(full, a @ b)),
            "gemv_ok": bool(torch.allclose(gemv(x, gather=True), x @ w.t())),
            "gemv_local_rows": gemv.w_local.shape[0],
        }
    except Exception as error:  # reported to the parent, never swallowed
        results[rank] = {"error": type(error).__name__ + ": " + str(error)[:200]}
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _decide(rank, world):
    """The collective choice of the gather form on CPU ranks."""

    import torch.distributed as dist

    from radeon_kernels.distributed.peer import fused_path_available
    from radeon_kernels.distributed.shard import ShardedGemv

    out = {"available": fused_path_available(torch.zeros(2, 2))}  # CPU tensors: every rank declines
    calls = []
    original = dist.all_gather_object

    def counting(*args, **kwargs):
        calls.append(1)
        return original(*args, **kwargs)

    dist.all_gather_object = counting
    try:
        auto = ShardedGemv(torch.randn(4 * world, 8), compute=None, fused=None)
        auto._compute = lambda p, q: p @ q.t()  # keep the NCCL form's plumbing on CPU
        auto._permute = _permute_cpu
        x = torch.randn(2, 8)
        for _ in range(3):
            auto(x, gather=True)
        out["decided_once"] = len(calls) == 1 and auto._fused is False
        required = ShardedGemv(torch.randn(4 * world, 8), fused=True)
        try:
            required(x, gather=True)
            out["required"] = "ran"
        except RuntimeError as error:
            out["required"] = "refused" if "NVLink" in str(error) else str(error)
    finally:
        dist.all_gather_object = original
    return out


def _run(world, mode="ok"):
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results, mode)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("rank did not finish")
    return dict(results)


def test_column_block_bounds():
    assert [(column_block(12, 3, r).start, column_block(12, 3, r).stop) for r in range(3)] == [(0, 4), (4, 8), (8, 12)]
    with pytest.raises(ValueError, match="not divisible"):
        column_block(10, 3, 0)
    with pytest.raises(ValueError, match="invalid rank"):
        column_block(12, 3, 3)


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_gemm_and_gemv_reassemble_the_full_result(world):
    results = _run(world)
    assert sorted(results) == list(range(world))
    for rank, res in results.items():
        assert "error" not in res, res
        assert res["block"] == (6 * rank, 6 * (rank + 1))
        assert res["local_ok"] and res["full_ok"] and res["gemv_ok"]
        assert res["gemv_local_rows"] == 4


def test_a_failing_rank_surfaces_as_errors_not_a_hang():
    results = _run(2, mode="fail")
    assert "error" in results[1]
    # rank 0 reaches the all-gather without its peer and fails on the short timeout
    assert "error" in results[0]


def test_the_gather_form_is_decided_once_and_together():
    """CPU ranks never take the fused peer-store path; the decision costs one collective call
    on the first gathered call only, and fused=True is refused on every rank alike."""

    results = _run(2, mode="decide")
    assert results == {r: {"available": False, "decided_once": True, "required": "refused"} for r in range(2)}, results
