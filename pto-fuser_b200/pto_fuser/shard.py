"""Data-parallel sharding of the GDN forward over the GPUs of one node.

Every (batch, head) pair is an independent recurrence (the reference's scan walks
(b, h) pairs independently, kernels/scan_fused.h:217; gdn_reference loops over them,
examples/attention/_gdn_full.py:65-66), so the job splits into contiguous blocks of
the B*H pairs, one block per rank, with no exchange on the data path. The only
collectives are the max-over-ranks step time and, when the caller wants the whole
result on one rank, a gather of the outputs.
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch


def shard_pairs(n_pairs: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [start, stop) block of the flattened (b, h) pairs owned by `rank`.
    Blocks differ in size by at most one pair; every pair is owned exactly once."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    base, extra = divmod(n_pairs, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_heads(x: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    """The rank's block of a [B, H, ...] tensor, flattened to [pairs, ...] (pairs in
    (b, h) order), contiguous."""
    B, H = x.shape[:2]
    a, b = shard_pairs(B * H, world, rank)
    return x.reshape(B * H, *x.shape[2:])[a:b].contiguous()


def max_over_ranks(value: float, device: Optional[torch.device] = None) -> float:
    """The largest of `value` over all ranks (the job's step time is its slowest rank's)."""
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], device=device or "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_pairs(local: torch.Tensor, n_pairs: int, dst: int = 0) -> Optional[torch.Tensor]:
    """Gather every rank's [pairs_r, ...] block into [n_pairs, ...] on rank `dst`
    (None elsewhere). Blocks may differ in size by one pair; they are padded to the
    largest block for the collective and trimmed on `dst`."""
    import torch.distributed as dist
    world, rank = dist.get_world_size(), dist.get_rank()
    sizes = [shard_pairs(n_pairs, world, r) for r in range(world)]
    cap = max(b - a for a, b in sizes)
    buf = torch.zeros((cap,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    buf[: local.shape[0]] = local
    parts: Optional[List[torch.Tensor]] = None
    if rank == dst:
        parts = [torch.empty_like(buf) for _ in range(world)]
    dist.gather(buf, parts, dst=dst)
    if rank != dst:
        return None
    return torch.cat([p[: b - a] for p, (a, b) in zip(parts, sizes)], dim=0)
