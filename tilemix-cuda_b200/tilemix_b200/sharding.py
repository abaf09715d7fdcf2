"""Host-side multi-GPU logic: batch x head sharding with no data-path collective.

Every (batch, head) slab is an independent attention problem and its output
stays on the GPU that computed it, so ranks never exchange data. Two modes:

* weak scaling (default in bench.py): every rank runs a full batch of heads of
  the configuration, drawn with its own seed; the job's work grows with N.
* strong scaling: one fixed batch of `total` heads is split into contiguous
  per-rank shards (the BASELINE configs' "heads sharded across 1/2/4/8 GPUs").

The only collectives are the start/stop barriers of a timed region and the
max-over-ranks reduction of device times (job time = slowest rank).
"""
from __future__ import annotations


def shard_heads(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, start + count) slice of `total` heads for `rank`;
    the first total % world ranks get one extra head."""
    if world <= 0 or not 0 <= rank < world or total < 0:
        raise ValueError("bad shard request")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def rank_seed(base_seed: int, rank: int) -> int:
    """Seed of a rank's inputs under weak scaling (rank 0 keeps the config's seed)."""
    return base_seed + 1000 * rank


def max_over_ranks(value: float, world: int, device=None) -> float:
    """Max of a per-rank float over the default process group (the job's time
    is its slowest rank). `device`: where the reduction tensor lives (cuda for
    NCCL, cpu for gloo)."""
    if world == 1:
        return float(value)
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(value)], dtype=torch.float64, device=device or "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, world: int, device=None) -> float:
    if world == 1:
        return float(value)
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(value)], dtype=torch.float64, device=device or "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())
