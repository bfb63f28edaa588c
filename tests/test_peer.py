"""Host logic of the NVLink peer gather (laplacianformer_b200.peer) on CPU:
buffer layout, the IPC-handle exchange over a world_size-2 gloo group and
the peer addresses each rank's kernels would store to, with the C-ABI calls
replaced by a recording fake (no GPU)."""
import torch
import torch.distributed as dist

from laplacianformer_b200.peer import PeerGather, layout
from test_sharding import _init, _run_pair

FAKE_BASE = 1 << 40


class FakeOps:
    """Buffers are host tensors; a rank's 'device address' is FAKE_BASE * (rank + 1)."""

    def __init__(self, rank):
        self.rank = rank
        self.opened, self.closed, self.freed, self.barriers = [], [], [], []

    def alloc(self, nbytes):
        self.nbytes = nbytes
        return FAKE_BASE * (self.rank + 1), bytes([self.rank]) * 64

    def open(self, handle):
        assert len(handle) == 64
        self.opened.append(handle[0])
        return FAKE_BASE * (handle[0] + 1)

    def close(self, ptr):
        self.closed.append(ptr)

    def free(self, ptr):
        self.freed.append(ptr)

    def barrier(self, flag_ptrs, rank, epoch, timeout_ms, stream):
        self.barriers.append((tuple(flag_ptrs), rank, epoch))

    def tensor(self, ptr, nbytes, device):
        return torch.zeros(nbytes, dtype=torch.uint8)


def test_layout_alignment_and_padding():
    outs = [((16384, 64), torch.bfloat16), ((64, 256), torch.bfloat16), ((256, 256), torch.float32)]
    offs, sizes, blocks, chunk, total = layout(outs, 127, 8)
    assert chunk == 16
    assert all(o % 256 == 0 for o in offs) and offs[0] >= 256 and total % 256 == 0
    assert blocks == [16 * 16384 * 64 * 2, 16 * 64 * 256 * 2, 16 * 256 * 256 * 4]
    assert sizes == [8 * b for b in blocks]
    for (o0, s0), o1 in zip(zip(offs, sizes), offs[1:]):
        assert o1 >= o0 + s0


def _peer_worker(rank, world, port, result_q):
    _init(rank, world, port)
    try:
        ops = FakeOps(rank)
        pg = PeerGather([((5, 3), torch.float16), ((7,), torch.float32)], total_bh=5, device="cpu", ops=ops)
        ok = pg.chunk == 3 and pg.gathered(0).shape == (6, 5, 3) and pg.gathered(1).dtype == torch.float32
        ok = ok and pg.local(0).shape == (3, 5, 3)
        other = 1 - rank
        ok = ok and ops.opened == [other]
        ok = ok and pg.peer_ptrs(0) == [FAKE_BASE * (other + 1) + pg.offs[0] + rank * 3 * 15 * 2]
        ok = ok and pg.peer_ptrs(1) == [FAKE_BASE * (other + 1) + pg.offs[1] + rank * 3 * 7 * 4]
        pg.gathered(1).view(2, 3, 7)[:, :, 0] = torch.arange(6, dtype=torch.float32).view(2, 3)
        ok = ok and pg.trimmed(1).shape == (5, 7) and pg.trimmed(1)[:, 0].tolist() == [0, 1, 2, 3, 4]
        pg.barrier(stream=object())
        pg.barrier(stream=object())
        ok = ok and [b[2] for b in ops.barriers] == [1, 2]
        ok = ok and ops.barriers[0][0] == (FAKE_BASE, 2 * FAKE_BASE) and ops.barriers[0][1] == rank
        pg.close()
        ok = ok and ops.closed == [FAKE_BASE * (other + 1)] and ops.freed == [FAKE_BASE * (rank + 1)]
        result_q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


def test_peer_gather_two_gloo_ranks():
    assert _run_pair(_peer_worker) == {0: True, 1: True}
