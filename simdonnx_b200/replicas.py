"""Batch-sharded replicas across GPUs (one process per GPU, no collective on the data path).

Images are independent, so a global batch is split into contiguous per-rank slices; every rank
runs its own session (context, arena, CUDA graph) on its slice. The only collectives are for
timing (a barrier, and the max over ranks of a measured time) and, when the caller wants the whole
result on one rank, a gather of the per-rank outputs.
"""
from __future__ import annotations

import numpy as np


def shard_range(global_batch: int, world: int, rank: int) -> tuple[int, int]:
    """[begin, end) of the images rank `rank` owns: contiguous slices, sizes differing by <= 1."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world / rank")
    base, extra = divmod(global_batch, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def max_over_ranks(value: float, dist=None, device=None) -> float:
    """Max of a per-rank scalar (a step time) over the process group; the value itself when alone."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device or "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_outputs(local: np.ndarray, dist=None) -> np.ndarray | None:
    """Concatenate the per-rank output slices in rank order on rank 0 (None on the other ranks)."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return local
    parts = [None] * dist.get_world_size()
    dist.all_gather_object(parts, local)
    return np.concatenate(parts, axis=0) if dist.get_rank() == 0 else None


class ShardFailure(RuntimeError):
    """Raised on rank 0 when one or more ranks' shards failed: `failed` maps rank -> message and
    `partial` holds the outputs of the ranks that succeeded (None for the failed ones), in rank
    order. The batch as a whole reports the failure; the other shards' results are not lost."""

    def __init__(self, failed: dict, partial: list):
        super().__init__("shard failure on rank(s) " + ", ".join(f"{r}: {m}" for r, m in sorted(failed.items())))
        self.failed = failed
        self.partial = partial


def run_shards(run_local, dist=None):
    """Runs this rank's shard (run_local() -> np.ndarray) and gathers every rank's status and
    output on rank 0. An exception inside run_local is caught on its own rank and reported, so every
    rank still takes the same collective step (no rank is left waiting). Rank 0 returns the
    concatenation in rank order when every shard succeeded and raises ShardFailure otherwise; the
    other ranks return None. A rank that dies instead of reporting ends rank 0's gather with the
    process group's error (its timeout bounds the wait)."""
    try:
        out, status = run_local(), None
    except Exception as e:  # reported to rank 0 below, never swallowed
        out, status = None, f"{type(e).__name__}: {e}"
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        if status is not None:
            raise ShardFailure({0: status}, [None])
        return out
    parts = [None] * dist.get_world_size()
    dist.all_gather_object(parts, (status, out))
    if dist.get_rank() != 0:
        return None
    failed = {r: s for r, (s, _) in enumerate(parts) if s is not None}
    if failed:
        raise ShardFailure(failed, [o for _, o in parts])
    return np.concatenate([o for _, o in parts], axis=0)
