"""N-column sharded GEMM/GEMV on 2..8 GPUs (one process per GPU), through the public API.

Each rank computes its column block with this library's kernels.  Both ways of assembling
the full result -- the fused kernels that store every block into every rank's output over
peer memory (``rk_gemm_allgather`` / ``rk_gemv_allgather``) and the NCCL all-gather plus
``rk_gather_column_blocks`` -- must reproduce the single-GPU product bit for bit (every
output element is accumulated in the same order whatever the column tiling), and sampled
rows must match the C oracle within the north-star tolerance.

BASELINE config 5 (A[16384, 8192] @ B[8192, 57344] bf16, uniform[-1, 1)/16, seed 4 on the
CPU generator) runs at every world size from 2 to the number of visible GPUs (at most 8).
"""

from __future__ import annotations

import os
import socket
import sys
import traceback
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _bits(t):
    import torch

    return t.contiguous().view(torch.int16)


def _scenario_config5(rank, world, torch, dist):
    """BASELINE config 5, B split into `world` column blocks."""

    import numpy as np

    import radeon_kernels as rk
    from gpu_util import seeded, to_bits
    from oracle import oracle
    from radeon_kernels.distributed import ShardedGemm

    gen = torch.Generator().manual_seed(4)
    a_cpu = seeded((16384, 8192), 4, "uniform16", "bf16", gen)
    b_cpu = seeded((8192, 57344), 4, "uniform16", "bf16", gen)
    nb = 57344 // world
    a = a_cpu.cuda()
    b_block = b_cpu[:, rank * nb : (rank + 1) * nb].contiguous().cuda()
    b_full = b_cpu.cuda()
    full = rk.gemm(a, b_full)
    del b_full
    fused = ShardedGemm(b_block, n_total=57344, fused=True)
    c_fused = fused(a, gather=True)
    torch.cuda.synchronize()
    same_fused = bool(torch.equal(_bits(full), _bits(c_fused)))
    c_nccl = ShardedGemm(b_block, n_total=57344, fused=False)(a, gather=True)
    torch.cuda.synchronize()
    same_nccl = bool(torch.equal(_bits(full), _bits(c_nccl)))
    del c_nccl
    if rank == 0:  # the oracle on rows 0, M-1 and six seeded rows of the gathered C
        rows = [0, 16383] + sorted(np.random.default_rng(4).choice(16384, 6, replace=False).tolist())
        o_bits, o32 = oracle.gemm(to_bits(a_cpu[rows]), to_bits(b_cpu), "bf16")
        oracle.assert_parity(to_bits(c_fused[rows]), o_bits, o32, "bf16")
    status = int(rk_status())
    fused.close()
    return {"fused_equal": same_fused, "nccl_equal": same_nccl, "status": status}


def _scenario_repeated(rank, world, torch, dist):
    """Back-to-back fused calls on one exchange (epochs advance, no stale blocks) for GEMM and
    GEMV at several M, each checked against the single-GPU kernel right after its call."""

    from gpu_util import seeded, to_bits
    from oracle import oracle
    from radeon_kernels import _native
    from radeon_kernels.distributed import ShardedGemm, ShardedGemv

    ext = _native.extension()
    gen = torch.Generator().manual_seed(11)
    n, k = 4096 * world, 1024
    b_cpu = seeded((k, n), 11, "uniform16", "bf16", gen)
    nb = n // world
    b_block = b_cpu[:, rank * nb : (rank + 1) * nb].contiguous().cuda()
    b_full = b_cpu.cuda()
    gemm = ShardedGemm(b_block, n_total=n, fused=True)
    gemm_ok = []
    for i in range(4):
        a = seeded((1024 + 256 * (i % 2), k), 20 + i, "uniform16", "bf16").cuda()  # two exchanges, alternating
        got = gemm(a, gather=True).clone()
        want = ext.gemm_out(a, b_full, torch.empty(a.shape[0], n, dtype=a.dtype, device="cuda"), _native.GEMM_VARIANTS["tc_2sm"])
        gemm_ok.append(bool(torch.equal(_bits(got), _bits(want))))
    gemm.close()

    w_cpu = seeded((8192, 8192), 1, "normal/8192", "bf16", torch.Generator().manual_seed(1))
    rows = 8192 // world
    w_block = w_cpu[rank * rows : (rank + 1) * rows].contiguous().cuda()
    w_full = w_cpu.cuda()
    gemv = ShardedGemv(w_block, n_total=8192, fused=True)
    gemv_ok, gemv_oracle = [], []
    for i, m in enumerate([1, 1, 4, 16, 1, 32]):
        x_cpu = seeded((m, 8192), 30 + i, "normal", "bf16")
        x = x_cpu.cuda()
        got = gemv(x, gather=True).clone()
        want = ext.gemv_out(x, w_full, torch.empty(m, 8192, dtype=x.dtype, device="cuda"), _native.GEMV_VARIANTS["stream"])
        gemv_ok.append(bool(torch.equal(_bits(got), _bits(want))))
        if rank == 0 and i < 4:
            o_bits, o32 = oracle.gemv(to_bits(x_cpu), to_bits(w_cpu), "bf16")
            oracle.assert_parity(to_bits(got), o_bits, o32, "bf16")
            gemv_oracle.append(True)
    gemv.close()
    return {"gemm": gemm_ok, "gemv": gemv_ok, "gemv_oracle": rank != 0 or len(gemv_oracle) == 4,
            "status": int(rk_status())}


def rk_status() -> int:
    from radeon_kernels import _native

    return _native.extension().device_status()


SCENARIOS = {"config5": _scenario_config5, "repeated": _scenario_repeated}


def _worker(rank, world, port, scenario, results):
    import datetime

    sys.path.insert(0, str(REPO / "radeon-kernels_b200"))
    sys.path.insert(0, str(REPO))
    sys.path.insert(0, str(REPO / "tests"))
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        results[rank] = SCENARIOS[scenario](rank, world, torch, dist)
        dist.barrier()
    except Exception as error:  # noqa: BLE001 -- reported to the parent
        results[rank] = {"error": repr(error)[:300], "trace": traceback.format_exc()[-1500:]}
    finally:
        dist.destroy_process_group()


def _run(world: int, scenario: str) -> dict:
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, scenario, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    alive = [p.pid for p in procs if p.is_alive()]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert not alive, f"ranks still running after 600 s: {alive}"
    return dict(results)


def _world_sizes() -> list[int]:
    import torch

    count = min(torch.cuda.device_count(), 8) if torch.cuda.is_available() else 0
    return [w for w in (2, 4, 8) if w <= count] or [2]


@pytest.mark.parametrize("world", _world_sizes())
def test_config5_sharded_gemm_matches_single_gpu(world):
    import torch

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    results = _run(world, "config5")
    expected = {"fused_equal": True, "nccl_equal": True, "status": 0}
    assert results == {r: expected for r in range(world)}, results


def test_fused_allgather_repeated_calls():
    import torch

    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs 2 GPUs")
    results = _run(world, "repeated")
    expected = {"gemm": [True] * 4, "gemv": [True] * 6, "gemv_oracle": True, "status": 0}
    assert results == {r: expected for r in range(world)}, results
