"""N-column sharding of GEMM / GEMV weights across the GPUs of one node.

No counterpart in the reference (it is single-GPU throughout).  The layout:

* GEMM  ``C[M,N] = A[M,K] @ B[K,N]``: rank g owns the column block ``B[:, g*N/G:(g+1)*N/G]``
  and computes ``C_g = A @ B_g`` -- independent blocks, no reduction.
* GEMV  ``out[M,N] = x[M,K] @ W[N,K]^T``: rank g owns the row block ``W[g*N/G:(g+1)*N/G, :]``
  and computes ``out_g``.
* Only when the caller needs the full result (``gather=True``), two ways to assemble it:

  - fused (default on NVLink-connected GPUs): one kernel per rank computes its block and
    stores it straight into every rank's full output through CUDA IPC peer pointers
    (``rk_gemm_allgather`` / ``rk_gemv_allgather``), so the exchange overlaps the math tile
    by tile and needs no collective call and no permute pass.  The result lives in a
    per-shape exchange buffer that the next gathered call with the same M rewrites (copy
    it to keep it);
  - NCCL: the local product, an ``all_gather_into_tensor`` of the per-rank blocks into
    ``[G, M, N/G]``, and ``rk_gather_column_blocks`` permuting them into row-major ``[M, N]``
    (CPU ``gloo`` groups, or ``fused=False``).

One process per GPU, ``torch.distributed`` for the process group.  The local products
run through the public ``radeon_kernels.gemm`` / ``radeon_kernels.gemv`` (dispatch ->
sm_100a kernels); ``compute``/``permute`` are injectable so the collective plumbing can be
exercised on CPU ``gloo`` ranks in tests (injecting them selects the NCCL form).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable


@dataclass(frozen=True)
class ColumnBlock:
    rank: int
    world: int
    start: int
    stop: int

    @property
    def size(self) -> int:
        return self.stop - self.start


def column_block(n: int, world: int, rank: int) -> ColumnBlock:
    """Equal contiguous blocks; ``n`` must be a multiple of ``world``."""

    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"invalid rank {rank} of world {world}")
    if n % world != 0:
        raise ValueError(f"N={n} is not divisible by the world size {world}")
    width = n // world
    return ColumnBlock(rank=rank, world=world, start=rank * width, stop=(rank + 1) * width)


def _dist() -> Any:
    import torch.distributed as dist

    return dist


def _default_permute(blocks: Any, out: Any) -> Any:
    from radeon_kernels import _native

    return _native.extension().gather_column_blocks(blocks, out)


def all_gather_columns(
    local: Any,
    *,
    group: Any = None,
    permute: Callable[[Any, Any], Any] | None = None,
    out: Any | None = None,
) -> Any:
    """All-gather per-rank column blocks ``local[M, N/G]`` into the full ``[M, N]``."""

    import torch

    dist = _dist()
    world = dist.get_world_size(group)
    m, nb = local.shape
    if world == 1:
        if out is None:
            return local
        out.copy_(local)
        return out
    # Concatenated [G*M, N/G] output (accepted by NCCL and gloo), viewed as [G, M, N/G].
    staged = torch.empty((world * m, nb), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(staged, local.contiguous(), group=group)
    staged = staged.view(world, m, nb)
    full = out if out is not None else torch.empty((m, world * nb), dtype=local.dtype, device=local.device)
    (permute or _default_permute)(staged, full)
    return full


class _FusedGather:
    """The fused compute + all-gather form shared by ShardedGemm and ShardedGemv.

    ``fused``: None = decide collectively on the first gathered call (every rank on its own
    NVLink-reachable GPU); True = require it; False = always the NCCL all-gather.
    """

    def _init_fused(self, fused: bool | None, injected: bool) -> None:
        self._required = fused is True
        # None until the first gathered call decides (collectively); then fixed, so later
        # calls make no collective call and can be captured into a CUDA graph.
        self._fused: bool | None = False if (injected or fused is False) else None
        self._exchanges: dict[tuple[int, Any], Any] = {}

    def _use_fused(self, operand: Any) -> bool:
        if self._fused is None:
            from radeon_kernels.distributed.peer import fused_path_available

            available = fused_path_available(operand, group=self.group)
            if self._required and not available:
                raise RuntimeError("the fused all-gather needs every rank on its own NVLink-connected GPU")
            self._fused = available
        return self._fused

    def _exchange(self, m: int, dtype: Any) -> Any:
        key = (m, dtype)
        exchange = self._exchanges.get(key)
        if exchange is None:
            from radeon_kernels.distributed.peer import PeerExchange

            exchange = PeerExchange((m, self.n_total), dtype, group=self.group)
            self._exchanges[key] = exchange
        return exchange

    def close(self) -> None:
        """Collective: releases the peer mappings of the fused form."""

        for exchange in self._exchanges.values():
            exchange.close()
        self._exchanges.clear()


def _aligned(t: Any) -> Any:
    # The fused kernels read 16-byte vectors; a misaligned view gets a fresh (aligned) copy on
    # every rank alike rather than a different kernel on one rank.
    t = t.contiguous()
    return t if t.data_ptr() % 16 == 0 else t.clone()


class ShardedGemm(_FusedGather):
    """``C = A @ B`` with B split by N-column blocks over the ranks of ``group``."""

    def __init__(
        self,
        b_full_or_block: Any,
        *,
        n_total: int | None = None,
        group: Any = None,
        compute: Callable[[Any, Any], Any] | None = None,
        permute: Callable[[Any, Any], Any] | None = None,
        fused: bool | None = None,
    ) -> None:
        dist = _dist()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self._init_fused(fused, compute is not None or permute is not None)
        if n_total is None:  # the full B was given: keep this rank's block only
            n_total = int(b_full_or_block.shape[1])
            self.block = column_block(n_total, self.world, self.rank)
            self.b_local = b_full_or_block[:, self.block.start : self.block.stop].contiguous()
        else:
            self.block = column_block(n_total, self.world, self.rank)
            if int(b_full_or_block.shape[1]) != self.block.size:
                raise ValueError("local B block has the wrong number of columns")
            self.b_local = b_full_or_block
        self.n_total = n_total
        if compute is None:
            import radeon_kernels as rk

            compute = rk.gemm
        self._compute = compute
        self._permute = permute

    def local(self, a: Any) -> Any:
        """This rank's ``C[:, start:stop]`` (no communication)."""

        return self._compute(a, self.b_local)

    def __call__(self, a: Any, *, gather: bool = False) -> Any:
        if gather and self.world > 1 and self._fusable(a) and self._use_fused(a):
            from radeon_kernels import _native

            a = _aligned(a)
            ex = self._exchange(int(a.shape[0]), a.dtype)
            return _native.extension().gemm_allgather(a, self.b_local, ex.output, ex.out_ptrs, ex.ctl_ptrs,
                                                      ex.rank, ex.timeout_ns)
        c_local = self.local(a)
        if not gather:
            return c_local
        return all_gather_columns(c_local, group=self.group, permute=self._permute)

    def _fusable(self, a: Any) -> bool:
        # The same answer on every rank: it depends only on shapes and dtypes.
        return (getattr(a, "dim", lambda: 0)() == 2 and a.shape[0] > 0 and a.shape[1] == self.b_local.shape[0]
                and a.dtype == self.b_local.dtype and self.block.size % 8 == 0 and a.shape[1] % 8 == 0
                and self.b_local.is_contiguous())


class ShardedGemv(_FusedGather):
    """``out = x @ W^T`` with W split by N-row blocks over the ranks of ``group``."""

    def __init__(
        self,
        w_full_or_block: Any,
        *,
        n_total: int | None = None,
        group: Any = None,
        compute: Callable[[Any, Any], Any] | None = None,
        permute: Callable[[Any, Any], Any] | None = None,
        fused: bool | None = None,
    ) -> None:
        dist = _dist()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self._init_fused(fused, compute is not None or permute is not None)
        if n_total is None:
            n_total = int(w_full_or_block.shape[0])
            self.block = column_block(n_total, self.world, self.rank)
            self.w_local = w_full_or_block[self.block.start : self.block.stop].contiguous()
        else:
            self.block = column_block(n_total, self.world, self.rank)
            if int(w_full_or_block.shape[0]) != self.block.size:
                raise ValueError("local W block has the wrong number of rows")
            self.w_local = w_full_or_block
        self.n_total = n_total
        if compute is None:
            import radeon_kernels as rk

            compute = rk.gemv
        self._compute = compute
        self._permute = permute

    def local(self, x: Any) -> Any:
        return self._compute(x, self.w_local)

    def __call__(self, x: Any, *, gather: bool = False) -> Any:
        if gather and self.world > 1 and self._fusable(x) and self._use_fused(x):
            from radeon_kernels import _native

            x = _aligned(x)
            ex = self._exchange(int(x.shape[0]), x.dtype)
            return _native.extension().gemv_allgather(x, self.w_local, ex.output, ex.out_ptrs, ex.ctl_ptrs,
                                                      ex.rank, ex.timeout_ns)
        out_local = self.local(x)
        if not gather:
            return out_local
        return all_gather_columns(out_local, group=self.group, permute=self._permute)

    def _fusable(self, x: Any) -> bool:
        # The same answer on every rank: it depends only on shapes and dtypes.
        return (getattr(x, "dim", lambda: 0)() == 2 and 1 <= x.shape[0] <= 32 and x.shape[1] == self.w_local.shape[1]
                and x.dtype == self.w_local.dtype and x.shape[1] % 8 == 0 and self.w_local.is_contiguous())


__all__ = ["ColumnBlock", "ShardedGemm", "ShardedGemv", "all_gather_columns", "column_block"]
