"""Multi-GPU sharding of the hot-path ops: one process per GPU, no collective on the hot path.

Every op family partitions into independent work units (the reference has no
distributed code; the partition follows the op's independence):

* row families (vector add, cumsum, softmax, RMSNorm): contiguous row blocks per rank;
* GEMM: contiguous M-panels of A and C per rank, B (and a bias[N]) replicated;
* attention: contiguous (batch, head) slices per rank.

Each rank generates / holds only its shard and launches the same kernel on it.
``gather_rows`` (NCCL all-gather over NVLink, or gloo on CPU) assembles a full output
for verification only — it is never inside a timed region.
"""

from __future__ import annotations

import os


def shard_bounds(total: int, rank: int, world: int) -> tuple[int, int]:
    """[begin, end) of ``rank``'s contiguous share of ``total`` units (sizes differ by <= 1)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(total, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def shard_rows(tensor, rank: int, world: int):
    """Rank's contiguous block of rows (dim 0), as a view."""
    b, e = shard_bounds(int(tensor.shape[0]), rank, world)
    return tensor[b:e]


def shard_heads(tensor, rank: int, world: int):
    """Rank's contiguous share of the flattened (batch, head) pairs of a [B, H, S, D] tensor,
    returned as [pairs, 1, S, D] (each (b, h) pair is an independent attention problem)."""
    B, H, S, D = tensor.shape
    flat = tensor.reshape(B * H, 1, S, D)
    b, e = shard_bounds(B * H, rank, world)
    return flat[b:e]


def gather_rows(local, world: int, group=None):
    """All-gather equal-or-ragged row shards into the full tensor (verification only)."""
    import torch
    import torch.distributed as dist

    counts = [None] * world
    dist.all_gather_object(counts, int(local.shape[0]), group=group)
    cap = max(counts)
    pad = torch.zeros((cap,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    return torch.cat([p[:c] for p, c in zip(parts, counts)], dim=0)


def env_rank_world() -> tuple[int, int, int]:
    """(rank, world_size, local_rank) from torchrun's environment (1 process when absent)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


__all__ = ["env_rank_world", "gather_rows", "shard_bounds", "shard_heads", "shard_rows"]
