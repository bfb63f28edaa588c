"""B*H sharding of both operators across ranks.

Every (b, h) slice of LaplaceSubtraction and every matrix of NewtonInverse is
independent, so rank r of W owns the contiguous slice
[start(r), start(r+1)) of the flattened leading B*H dimension (the leading
dimensions are the outermost, so a slice is one contiguous block of memory)
and computes it with no communication.  Where a caller needs the outputs
replicated, :func:`all_gather_bh` assembles them with one
``all_gather_into_tensor`` per output (NCCL over NVLink on GPUs, gloo on
CPU); uneven splits are padded to the largest slice and trimmed.
"""
from __future__ import annotations

from typing import Callable, Sequence

import torch
import torch.distributed as dist


def shard_bounds(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced split of `total` units: the first total % world
    ranks get one extra unit."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError("bad world/rank")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def flatten_bh(t: torch.Tensor) -> torch.Tensor:
    """[B, H, ...] -> [B*H, ...] (a view for contiguous tensors)."""
    return t.reshape(t.shape[0] * t.shape[1], *t.shape[2:])


def local_slice(t: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    """This rank's contiguous [bh_local, ...] block of a [B, H, ...] tensor."""
    f = flatten_bh(t)
    s, e = shard_bounds(f.shape[0], world, rank)
    return f[s:e]


def all_gather_bh(local: torch.Tensor, total_bh: int, group=None) -> torch.Tensor:
    """Gather every rank's [bh_r, ...] block into [total_bh, ...] on all ranks."""
    world = dist.get_world_size(group)
    chunk = -(-total_bh // world)  # every rank sends an equal, padded block
    send = local
    if local.shape[0] != chunk:
        send = local.new_zeros((chunk,) + tuple(local.shape[1:]))
        send[: local.shape[0]] = local
    out = local.new_empty((chunk * world,) + tuple(local.shape[1:]))
    dist.all_gather_into_tensor(out, send.contiguous(), group=group)
    if total_bh % world == 0:
        return out
    parts = []
    for r in range(world):
        s, e = shard_bounds(total_bh, world, r)
        parts.append(out[r * chunk: r * chunk + (e - s)])
    return torch.cat(parts, 0)


def run_sharded(fn: Callable[..., Sequence[torch.Tensor]], inputs: Sequence[torch.Tensor], gather: bool = True,
                group=None) -> list[torch.Tensor]:
    """Apply `fn` to this rank's B*H slice of every input ([B, H, ...]
    tensors sharing B*H) and optionally all-gather the outputs.

    `fn` receives the local blocks as [1, bh_local, ...] tensors and returns
    [1, bh_local, ...] outputs.  Gathered outputs come back as [B*H, ...];
    ungathered ones as the local [bh_local, ...] blocks.
    """
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    total = inputs[0].shape[0] * inputs[0].shape[1]
    for t in inputs:
        if t.shape[0] * t.shape[1] != total:
            raise ValueError("inputs must share B*H")
    local = [local_slice(t, world, rank).unsqueeze(0) for t in inputs]
    outs = [flatten_bh(o) for o in fn(*local)]
    if not gather or world == 1:
        return outs
    return [all_gather_bh(o, total, group) for o in outs]
