"""Batch sharding over ranks (one process per GPU) and the host-side collectives around it.

The conv / bmm path shards on the batch dimension: images (or bmm batch items) are independent,
weights are replicated, and no collective touches the data path.  Collectives run only after the
timed region: the max over ranks of the measured times, and a gather of per-rank results for
verification.  Works with any torch.distributed backend (NCCL on GPUs, gloo on CPU).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(total: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous, balanced share of `total` items for `rank`: (start, count)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def world_info() -> tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def max_over_ranks(values, device=None) -> list[float]:
    """Element-wise max of a list of floats over all ranks (identity without a process group)."""
    vals = [float(v) for v in values]
    rank, world = world_info()
    if world == 1:
        return vals
    t = torch.tensor(vals, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def gather_tensors(t: torch.Tensor) -> list[torch.Tensor]:
    """All-gather of a same-shaped tensor from every rank (verification only, untimed)."""
    rank, world = world_info()
    if world == 1:
        return [t]
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t.contiguous())
    return out


def checksum(t: torch.Tensor) -> torch.Tensor:
    """Order-independent checksum of a tensor's bytes (sum of unsigned bytes, int64)."""
    return t.contiguous().view(torch.uint8).to(torch.int64).sum().reshape(1)
