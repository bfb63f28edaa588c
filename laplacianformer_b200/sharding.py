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


def run_sharded_overlapped(fn: Callable[..., Sequence[torch.Tensor]], inputs: Sequence[torch.Tensor],
                           chunks: int = 4, group=None) -> list[torch.Tensor]:
    """run_sharded(..., gather=True) with the all-gather overlapped with compute.

    This rank's B*H slice is cut into `chunks` pieces of c = ceil(ceil(B*H /
    world) / chunks) slices (every rank uses the same c, padding its last
    pieces).  Piece i is computed, then its outputs are all-gathered with an
    asynchronous collective while piece i+1 is computed (NCCL runs the
    gather on its own stream after the work already queued on the current
    stream; gloo on its own thread).  Returns the outputs as [B*H, ...], the
    same as run_sharded.
    """
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    total = inputs[0].shape[0] * inputs[0].shape[1]
    for t in inputs:
        if t.shape[0] * t.shape[1] != total:
            raise ValueError("inputs must share B*H")
    if world == 1:
        return run_sharded(fn, inputs, gather=False, group=group)
    local = [local_slice(t, world, rank) for t in inputs]
    n_local = local[0].shape[0]
    per_rank = -(-total // world)
    chunks = max(1, min(chunks, per_rank))
    c = -(-per_rank // chunks)
    pending = []  # (piece index, gathered buffers, works)
    for i in range(chunks):
        a, b = min(i * c, n_local), min((i + 1) * c, n_local)
        if b > a:
            outs = [flatten_bh(o) for o in fn(*[t[a:b].unsqueeze(0) for t in local])]
        else:  # this rank has no slices left for this piece: gather zeros
            shapes = pending[0][3] if pending else None
            if shapes is None:
                probe = fn(*[t[:1].unsqueeze(0) for t in local])
                shapes = [(tuple(o.shape[2:]), o.dtype, o.device) for o in probe]
            outs = [torch.zeros((0,) + s, dtype=dt, device=dv) for s, dt, dv in shapes]
        sends, bufs, works = [], [], []
        for o in outs:
            send = o
            if o.shape[0] != c:
                send = o.new_zeros((c,) + tuple(o.shape[1:]))
                send[: o.shape[0]] = o
            buf = o.new_empty((c * world,) + tuple(o.shape[1:]))
            works.append(dist.all_gather_into_tensor(buf, send.contiguous(), group=group, async_op=True))
            sends.append(send)
            bufs.append(buf)
        shapes = [(tuple(o.shape[1:]), o.dtype, o.device) for o in outs]
        pending.append((i, bufs, works, shapes, sends))
    for _, _, works, _, _ in pending:
        for w in works:
            w.wait()
    # assemble: rank r's piece i holds its slices [i*c, i*c + len) at global start(r) + i*c
    n_out = len(pending[0][1])
    result = []
    for k in range(n_out):
        ref = pending[0][1][k]
        out = ref.new_empty((total,) + tuple(ref.shape[1:]))
        for i, bufs, _, _, _ in pending:
            for r in range(world):
                s, e = shard_bounds(total, world, r)
                a, b = min(s + i * c, e), min(s + (i + 1) * c, e)
                if b > a:
                    out[a:b] = bufs[k][r * c: r * c + (b - a)]
        result.append(out)
    return result
