"""All-gather of a (b,h)-sharded run through NVLink peer memory.

Same result layout as :func:`laplacianformer_b200.sharding.all_gather_bh`
(rank r's block of ``chunk = ceil(B*H / world)`` slices at ``[r*chunk,
(r+1)*chunk)``), but instead of a collective after the compute, the kernels
that produce an output store it straight into every rank's gather buffer:

* each rank allocates ONE device buffer (``lf_peer_alloc``: flags, then one
  region per output) and the ranks exchange its CUDA IPC handle over the
  process group; every rank maps the others' buffers (``lf_peer_open``);
* :meth:`PeerGather.peer_ptrs` gives, for output k, the address of this
  rank's block inside every OTHER rank's buffer; the balanced backward
  (``capi.laplace_sub_bwd_peers``) stores dQ there as it computes it, and
  ``capi.peer_put`` pushes small outputs;
* :meth:`PeerGather.barrier` (``lf_peer_barrier``, stream-ordered, bounded
  wait) makes every rank's stores visible before later work on the stream
  reads the gathered tensors.

One process per GPU, all ranks on one node.  A step that overwrites the
buffers must not start on any rank before every rank has finished reading
the previous step's contents (the caller's barrier placement decides this;
a reader that only uses the data inside the same step, before the next
step's barrier, is safe).
"""
from __future__ import annotations

import ctypes
import math
from typing import Sequence

import torch
import torch.distributed as dist

from . import capi

_ALIGN = 256
_FLAG_BYTES = 256  # uint32 flag per rank (LF_MAX_PEERS + 1 ranks at most)


class _CudaOps:
    """The C-ABI calls PeerGather makes (swappable for host-only tests)."""

    def alloc(self, nbytes: int):
        ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(capi.LF_PEER_HANDLE_BYTES)
        capi._check(capi.lib().lf_peer_alloc(nbytes, ctypes.byref(ptr), handle), "lf_peer_alloc")
        return int(ptr.value), handle.raw

    def open(self, handle: bytes) -> int:
        ptr = ctypes.c_void_p()
        capi._check(capi.lib().lf_peer_open(handle, ctypes.byref(ptr)), "lf_peer_open")
        return int(ptr.value)

    def close(self, ptr: int) -> None:
        capi._check(capi.lib().lf_peer_close(ctypes.c_void_p(ptr)), "lf_peer_close")

    def free(self, ptr: int) -> None:
        capi._check(capi.lib().lf_peer_free(ctypes.c_void_p(ptr)), "lf_peer_free")

    def barrier(self, flag_ptrs: Sequence[int], rank: int, epoch: int, timeout_ms: int, stream) -> None:
        table = (ctypes.c_void_p * len(flag_ptrs))(*flag_ptrs)
        capi._check(capi.lib().lf_peer_barrier(table, len(flag_ptrs), rank, epoch & 0xFFFFFFFF, timeout_ms,
                                               ctypes.c_void_p(stream.cuda_stream)), "lf_peer_barrier")

    def tensor(self, ptr: int, nbytes: int, device) -> torch.Tensor:
        return torch.as_tensor(_DeviceBytes(ptr, nbytes), device=device)


class _DeviceBytes:
    """A uint8 view of raw device memory (__cuda_array_interface__)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}


def _round_up(x: int, a: int) -> int:
    return (x + a - 1) // a * a


def layout(outputs: Sequence[tuple[tuple[int, ...], torch.dtype]], total_bh: int, world: int):
    """(region offsets, region bytes, per-rank block bytes, chunk, total bytes) of the shared buffer:
    flags first, then output k as [world * chunk, *item_shape] of its dtype."""
    chunk = -(-total_bh // world)
    offs, sizes, blocks = [], [], []
    off = _FLAG_BYTES
    for item_shape, dtype in outputs:
        item = math.prod(item_shape) * torch.empty((), dtype=dtype).element_size()
        block = chunk * item
        off = _round_up(off, _ALIGN)
        offs.append(off)
        sizes.append(world * block)
        blocks.append(block)
        off += world * block
    return offs, sizes, blocks, chunk, _round_up(off, _ALIGN)


class PeerGather:
    """Gather buffers for `outputs` ((item_shape, dtype) per output, an item
    being one (b,h) slice) of a run whose `total_bh` slices are sharded with
    :func:`sharding.shard_bounds` over the ranks of `group`."""

    def __init__(self, outputs: Sequence[tuple[tuple[int, ...], torch.dtype]], total_bh: int, group=None,
                 device=None, ops=None, timeout_ms: int = 5000):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world > capi.LF_MAX_PEERS + 1:
            raise ValueError(f"at most {capi.LF_MAX_PEERS + 1} ranks")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.ops = ops or _CudaOps()
        self.outputs = [(tuple(s), d) for s, d in outputs]
        self.total_bh = total_bh
        self.timeout_ms = timeout_ms
        self.offs, self.sizes, self.blocks, self.chunk, self.nbytes = layout(self.outputs, total_bh, self.world)
        self.base, handle = self.ops.alloc(self.nbytes)
        self.bases = [0] * self.world
        self.bases[self.rank] = self.base
        self._opened = []
        self._views = []
        handles = [None] * self.world
        try:
            if self.world > 1:
                dist.all_gather_object(handles, handle, group=group)
        except Exception:
            self.close(wait_for_peers=False)
            raise
        err = None
        try:
            for r in range(self.world):
                if r != self.rank:
                    self.bases[r] = self.ops.open(handles[r])
                    self._opened.append(self.bases[r])
        except Exception as exc:  # agreed on below, so that every rank gives up together
            err = exc
        errs = [None] * self.world
        if self.world > 1:
            dist.all_gather_object(errs, None if err is None else repr(err), group=group)
        else:
            errs = [None if err is None else repr(err)]
        failed = [(r, e) for r, e in enumerate(errs) if e is not None]
        if failed:
            self.close()
            raise RuntimeError(f"peer mapping failed on rank(s) {failed}")
        self.epoch = 0
        raw = self.ops.tensor(self.base, self.nbytes, self.device)
        self._views = [raw[o:o + n].view(dtype).view((self.world * self.chunk,) + shape)
                       for o, n, (shape, dtype) in zip(self.offs, self.sizes, self.outputs)]

    def gathered(self, k: int) -> torch.Tensor:
        """Output k on this GPU: [world * chunk, *item_shape] (rank r's block at r * chunk)."""
        return self._views[k]

    def local(self, k: int) -> torch.Tensor:
        """This rank's block of output k ([chunk, *item_shape]): where its kernels write locally."""
        return self._views[k][self.rank * self.chunk:(self.rank + 1) * self.chunk]

    def peer_ptrs(self, k: int) -> list[int]:
        """Address of this rank's block of output k in every other rank's buffer."""
        off = self.offs[k] + self.rank * self.blocks[k]
        return [self.bases[r] + off for r in range(self.world) if r != self.rank]

    def flag_ptrs(self) -> list[int]:
        return list(self.bases)

    def barrier(self, stream=None) -> None:
        """Stream-ordered barrier over the ranks (no-op with one rank)."""
        if self.world == 1:
            return
        self.epoch += 1
        stream = stream or torch.cuda.current_stream(self.device)
        self.ops.barrier(self.flag_ptrs(), self.rank, self.epoch, self.timeout_ms, stream)

    def trimmed(self, k: int) -> torch.Tensor:
        """Output k as [total_bh, *item_shape] (padding of uneven splits removed; a copy if any)."""
        from .sharding import shard_bounds
        g = self._views[k]
        if self.total_bh == self.world * self.chunk:
            return g
        parts = []
        for r in range(self.world):
            s, e = shard_bounds(self.total_bh, self.world, r)
            parts.append(g[r * self.chunk:r * self.chunk + (e - s)])
        return torch.cat(parts, 0)

    def close(self, wait_for_peers: bool = True) -> None:
        """Unmaps the peers' buffers and frees this rank's, after a device
        synchronisation and (with `wait_for_peers`, the default) a host
        barrier, so that no peer still maps it.  A collective call: every rank
        closes."""
        if self.base is None:
            return
        if self.device.type == "cuda" and torch.cuda.is_available():
            torch.cuda.synchronize(self.device)
        for p in self._opened:
            self.ops.close(p)
        self._opened = []
        self._views = []
        if wait_for_peers and self.world > 1:
            dist.barrier(group=self.group)
        self.ops.free(self.base)
        self.base = None
