"""Batch sharding across ranks (one process per GPU).

Batch elements are independent iLQR problems, so rank r of W solves the
contiguous slice [lo, hi) of the batch with no communication. After the
solve, the results the caller consumes are gathered over torch.distributed
(NCCL on GPUs, gloo on CPU): the first controls U[:, 0, :] (the actions the
policy steps with) and, after the backward, the gradients (dL/dx0 by
default; dL/dc or dL/dC on request). The reference has no multi-GPU path; its
caller solves the whole batch in one process
(acmpc_public-master/training_modules/mlp_mpc_policy_diffmpc.py:324-399).
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


def gather_rows(x_local: torch.Tensor, B: int, group=None) -> torch.Tensor:
    """All-gather the per-element rows x_local [hi - lo, ...] of every rank's
    shard into one [B, ...] tensor, in batch order. Shards are padded to
    equal length for all_gather_into_tensor; every rank receives the result
    (rank 0 is the consumer)."""
    world = dist.get_world_size(group)
    tail = tuple(x_local.shape[1:])
    width = 1
    for d in tail:
        width *= d
    per = (B + world - 1) // world
    even = B % world == 0
    if even and x_local.is_contiguous():
        # equal shards: the rank's rows are sent as they are and the gathered
        # buffer is already in batch order (no padding, no reassembly copy)
        buf = x_local.reshape(per, width)
    else:
        buf = torch.zeros(per, width, device=x_local.device, dtype=x_local.dtype)
        buf[: x_local.shape[0]] = x_local.reshape(x_local.shape[0], width)
    out = torch.empty(per * world, width, device=x_local.device, dtype=x_local.dtype)
    dist.all_gather_into_tensor(out, buf, group=group)
    if even:
        return out.reshape((B,) + tail)
    parts = []
    for r in range(world):
        lo, hi = shard_bounds(B, r, world)
        parts.append(out[r * per: r * per + (hi - lo)])
    return torch.cat(parts, 0).reshape((B,) + tail)


def gather_first_actions(U_local: torch.Tensor, B: int, group=None) -> torch.Tensor:
    """All-gather U_local[:, 0, :] from every rank into a [B, nu] tensor."""
    return gather_rows(U_local[:, 0, :], B, group)


def gather_actions_and_gradients(U_local: torch.Tensor, grads: dict, B: int, keys=("x0",), group=None):
    """gather_first_actions and gather_gradients in one collective: the
    first controls and the per-element gradients `keys` are packed into one
    [hi - lo, nu + sum of widths] buffer per rank, all-gathered once, and
    unpacked. Returns (actions [B, nu], dict of [B, ...] gradients)."""
    parts = [U_local[:, 0, :]] + [grads[k].reshape(grads[k].shape[0], -1) for k in keys]
    packed = gather_rows(torch.cat(parts, 1), B, group)
    nu = U_local.shape[-1]
    acts = packed[:, :nu]
    out, col = {}, nu
    for k in keys:
        tail = tuple(grads[k].shape[1:])
        width = 1
        for d in tail:
            width *= d
        out[k] = packed[:, col:col + width].reshape((B,) + tail)
        col += width
    return acts, out


def gather_gradients(grads: dict, B: int, keys=("x0",), group=None) -> dict:
    """All-gather the per-element gradients `keys` of a rank's backward
    (the dict ilqr_native.backward returns, batch-major) into [B, ...]
    tensors: dL/dx0 [B, 10] by default, "c" [B, T, 14] or "C" [B, T, 14, 14]
    when the consumer lives on rank 0."""
    return {k: gather_rows(grads[k], B, group) for k in keys}
