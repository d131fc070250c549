"""N-column sharding of GEMM / GEMV weights across the GPUs of one node.

No counterpart in the reference (it is single-GPU throughout).  The layout:

* GEMM  ``C[M,N] = A[M,K] @ B[K,N]``: rank g owns the column block ``B[:, g*N/G:(g+1)*N/G]``
  and computes ``C_g = A @ B_g`` -- independent blocks, no reduction, no collective.
* GEMV  ``out[M,N] = x[M,K] @ W[N,K]^T``: rank g owns the row block ``W[g*N/G:(g+1)*N/G, :]``
  and computes ``out_g``.
* Only when the caller needs the full result: one NCCL all-gather of the per-rank blocks
  into ``[G, M, N/G]`` (NVLink/NVSwitch), then ``rk_gather_column_blocks`` permutes them
  into the row-major ``[M, N]`` matrix on each GPU (one HBM pass).

One process per GPU, ``torch.distributed`` for the process group.  The local products
run through the public ``radeon_kernels.gemm`` / ``radeon_kernels.gemv`` (dispatch ->
sm_100a kernels); ``compute``/``permute`` are injectable so the collective plumbing can be
exercised on CPU ``gloo`` ranks in tests.
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
        return local
    # Concatenated [G*M, N/G] output (accepted by NCCL and gloo), viewed as [G, M, N/G].
    staged = torch.empty((world * m, nb), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(staged, local.contiguous(), group=group)
    staged = staged.view(world, m, nb)
    full = out if out is not None else torch.empty((m, world * nb), dtype=local.dtype, device=local.device)
    (permute or _default_permute)(staged, full)
    return full


class ShardedGemm:
    """``C = A @ B`` with B split by N-column blocks over the ranks of ``group``."""

    def __init__(
        self,
        b_full_or_block: Any,
        *,
        n_total: int | None = None,
        group: Any = None,
        compute: Callable[[Any, Any], Any] | None = None,
        permute: Callable[[Any, Any], Any] | None = None,
    ) -> None:
        dist = _dist()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
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
        c_local = self.local(a)
        if not gather:
            return c_local
        return all_gather_columns(c_local, group=self.group, permute=self._permute)


class ShardedGemv:
    """``out = x @ W^T`` with W split by N-row blocks over the ranks of ``group``."""

    def __init__(
        self,
        w_full_or_block: Any,
        *,
        n_total: int | None = None,
        group: Any = None,
        compute: Callable[[Any, Any], Any] | None = None,
        permute: Callable[[Any, Any], Any] | None = None,
    ) -> None:
        dist = _dist()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
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
        out_local = self.local(x)
        if not gather:
            return out_local
        return all_gather_columns(out_local, group=self.group, permute=self._permute)


__all__ = ["ColumnBlock", "ShardedGemm", "ShardedGemv", "all_gather_columns", "column_block"]
