"""Batch sharding across ranks (one process per GPU).

Batch elements are independent iLQR problems, so rank r of W solves the
contiguous slice [lo, hi) of the batch with no communication; the only
collective is one all-gather of the first controls U[:, 0, :] (the actions
the policy consumes) after the solve, through torch.distributed (NCCL on
GPUs, gloo on CPU).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_bounds(B: int, rank: int, world: int):
    """Contiguous slice of B elements for `rank`; the first B % world ranks
    take one extra element."""
    base, extra = divmod(B, world)
    lo = rank * base + min(rank, extra)
    hi = lo + base + (1 if rank < extra else 0)
    return lo, hi


def gather_first_actions(U_local: torch.Tensor, B: int, group=None) -> torch.Tensor:
    """All-gather U_local[:, 0, :] from every rank into a [B, nu] tensor
    (shards padded to equal length for all_gather_into_tensor)."""
    world = dist.get_world_size(group)
    nu = U_local.shape[-1]
    per = (B + world - 1) // world
    buf = torch.zeros(per, nu, device=U_local.device, dtype=U_local.dtype)
    buf[: U_local.shape[0]] = U_local[:, 0, :]
    out = torch.empty(per * world, nu, device=U_local.device, dtype=U_local.dtype)
    dist.all_gather_into_tensor(out, buf, group=group)
    parts = []
    for r in range(world):
        lo, hi = shard_bounds(B, r, world)
        parts.append(out[r * per: r * per + (hi - lo)])
    return torch.cat(parts, 0)
