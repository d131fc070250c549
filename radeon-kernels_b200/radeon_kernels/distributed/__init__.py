"""Multi-GPU sharding of the hot path (N-column blocks, optional NCCL all-gather)."""

from radeon_kernels.distributed.shard import ColumnBlock, ShardedGemm, ShardedGemv, all_gather_columns, column_block

__all__ = ["ColumnBlock", "ShardedGemm", "ShardedGemv", "all_gather_columns", "column_block"]
