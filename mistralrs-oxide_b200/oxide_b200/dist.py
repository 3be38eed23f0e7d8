"""Row partitioning across GPUs and the one cross-GPU exchange of the path.

Every op of the hot path is independent per token row (RMSNorm, add, SiLU*mul,
argmax, RoPE per token, softmax per (batch, head, query) row), so rows are
split into contiguous blocks, one per rank, with no data-path communication;
broadcast operands (norm weights, row-broadcast scales, RoPE tables, KV
lengths) are replicated.  Only whole-tensor reductions (sum / max / sum of
squares) need an exchange: each rank reduces its block to one f64 partial with
oxide_reduce_*, and a single all-reduce of that one value (NCCL over NVLink on
GPUs, gloo on CPU) combines them.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ._lib import RED_MAX, RED_SUM, RED_SUMSQ


def row_range(rows: int, rank: int, world: int) -> tuple[int, int]:
    """[lo, hi) of the contiguous block of rows owned by `rank`; block sizes
    differ by at most one row and the blocks cover [0, rows) exactly once."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    base, extra = divmod(rows, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def combine_partial(partial: torch.Tensor, op: int, group=None) -> torch.Tensor:
    """All-reduce a rank's f64 partial of a whole-tensor reduction in place:
    sum for OXIDE_RED_SUM / OXIDE_RED_SUMSQ, max for OXIDE_RED_MAX."""
    if op not in (RED_SUM, RED_MAX, RED_SUMSQ):
        raise ValueError(f"unknown reduction {op}")
    if partial.dtype != torch.float64 or partial.numel() != 1:
        raise ValueError("a partial is one float64 value")
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(partial, op=dist.ReduceOp.MAX if op == RED_MAX else dist.ReduceOp.SUM,
                        group=group)
    return partial


def global_reduce(x_shard: torch.Tensor, op: int, group=None) -> torch.Tensor:
    """Whole-tensor reduction of a row-sharded tensor: this rank's shard is
    reduced on its GPU (oxide_reduce_*), then the partials are all-reduced."""
    from . import ops

    return combine_partial(ops.reduce(x_shard, op), op, group)
