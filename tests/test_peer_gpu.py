"""The peer-store gather on the GPU.

One GPU: the balanced wide backward storing dQ into extra destinations
(local buffers stand in for the peers' gather buffers), the put kernel, and
the barrier's release/acquire and bounded wait on flags in local memory.
Two GPUs (skipped with fewer): two NCCL ranks gather dQ, dK^T and X through
IPC-mapped peer buffers and check every block against a local recomputation
of that rank's shard."""
import ctypes
import os

import pytest
import torch

from laplacianformer_b200 import capi

pytestmark = pytest.mark.gpu


def _inputs(shape, dtype, seed, device):
    B, H, N, D, M = shape
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, N, D, generator=g).to(dtype).to(device)
    k = torch.randn(B, H, D, M, generator=g).to(dtype).to(device)
    gr = torch.randn(B, H, N, M, generator=g).to(dtype).to(device)
    return q, k, gr


@pytest.mark.parametrize("shape", [(1, 3, 700, 64, 256), (2, 2, 333, 40, 131), (2, 2, 300, 32, 49)], ids=str)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=str)
def test_backward_peer_stores_match_plain(cuda, shape, dtype):
    q, k, g = _inputs(shape, dtype, 5, cuda)
    ws = torch.empty(max(1, capi.laplace_sub_bwd_workspace_size(q, k)), dtype=torch.uint8, device=cuda)
    dq0, dk0 = capi.laplace_sub_bwd(g, q, k, workspace=ws)
    peers = [torch.full_like(q, float("nan")) for _ in range(3)]
    dq, dk = torch.empty_like(q), torch.empty_like(k)
    capi.laplace_sub_bwd_peers(g, q, k, dq, dk, [p.data_ptr() for p in peers], workspace=ws)
    torch.cuda.synchronize()
    assert torch.equal(dq, dq0) and torch.equal(dk, dk0)
    for p in peers:
        assert torch.equal(p, dq0)


@pytest.mark.parametrize("nbytes", [16, 4096 * 16, 1001])
def test_peer_put_copies_to_every_destination(cuda, nbytes):
    src = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, device=cuda)
    dsts = [torch.zeros(nbytes + 16, dtype=torch.uint8, device=cuda) for _ in range(capi.LF_MAX_PEERS)]
    capi.peer_put(src, [d.data_ptr() for d in dsts])
    torch.cuda.synchronize()
    for d in dsts:
        assert torch.equal(d[:nbytes], src) and int(d[nbytes:].sum()) == 0


def _barrier(flags, rank, epoch, timeout_ms):
    table = (ctypes.c_void_p * len(flags))(*[f.data_ptr() for f in flags])
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return capi.lib().lf_peer_barrier(table, len(flags), rank, epoch, timeout_ms, st)


def test_peer_barrier_signals_and_times_out(cuda):
    capi.device_status(clear=True)
    flags = [torch.zeros(16, dtype=torch.int32, device=cuda) for _ in range(2)]
    flags[0][1] = 1  # rank 1's signal for epoch 1 is already there
    assert _barrier(flags, 0, 1, 2000) == capi.LF_OK
    assert capi.device_status(clear=True) == capi.LF_OK
    assert int(flags[1][0]) == 1  # this rank's signal reached rank 1's array
    # epoch 2: nothing sets rank 1's signal, so the bounded wait expires
    assert _barrier(flags, 0, 2, 50) == capi.LF_OK
    assert capi.device_status(clear=True) == capi.LF_ERR_TIMEOUT
    assert int(flags[1][0]) == 2
    assert capi.device_status(clear=True) == capi.LF_OK
    assert _barrier(flags, 2, 3, 50) == capi.LF_ERR_INVALID  # rank outside the world


def _two_rank_worker(rank, world, port, result_q):
    import torch.distributed as dist

    from laplacianformer_b200.peer import PeerGather
    from laplacianformer_b200.sharding import shard_bounds

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        B, H, N, D, M = 1, 5, 600, 64, 256
        q, k, g = _inputs((B, H, N, D, M), torch.bfloat16, 9, dev)
        A = (torch.rand(B * H, 16, 16, generator=torch.Generator().manual_seed(4)) * 0.05 + torch.eye(16)).to(dev)
        pg = PeerGather([((N, D), q.dtype), ((D, M), k.dtype), ((16, 16), torch.float32)], B * H)
        s, e = shard_bounds(B * H, world, rank)
        ws = torch.empty(capi.laplace_sub_bwd_workspace_size(q[:, s:e], k[:, s:e]), dtype=torch.uint8, device=dev)
        fails = []
        for step in range(3):
            dq = pg.local(0)[: e - s].unsqueeze(0)
            dk = pg.local(1)[: e - s].unsqueeze(0)
            capi.laplace_sub_bwd_peers(g[:, s:e].contiguous(), q[:, s:e].contiguous(), k[:, s:e].contiguous(),
                                       dq, dk, pg.peer_ptrs(0), workspace=ws)
            capi.peer_put(pg.local(1)[: e - s], pg.peer_ptrs(1))
            X = pg.local(2)[: e - s]
            capi.newton_inverse_fwd(A[s:e].contiguous().unsqueeze(0), 8, out=X.unsqueeze(0))
            capi.peer_put(X, pg.peer_ptrs(2))
            pg.barrier()
            torch.cuda.synchronize()
            for r in range(world):
                a, b = shard_bounds(B * H, world, r)
                rdq, rdk = capi.laplace_sub_bwd(g[:, a:b].contiguous(), q[:, a:b].contiguous(),
                                                k[:, a:b].contiguous())
                rx = capi.newton_inverse_fwd(A[a:b].contiguous().unsqueeze(0), 8)
                c = pg.chunk
                for name, got, want in (("dq", pg.gathered(0), rdq), ("dk", pg.gathered(1), rdk),
                                        ("x", pg.gathered(2), rx)):
                    blk = got[r * c: r * c + b - a].float()
                    if not torch.equal(blk, want[0].float()):
                        fails.append((step, r, name, float((blk - want[0].float()).abs().max())))
            if pg.trimmed(0).shape != (B * H, N, D):
                fails.append((step, "trimmed shape"))
            dist.barrier()
        st = capi.device_status(clear=True)
        if st != capi.LF_OK:
            fails.append(("device status", st))
        pg.close()
        result_q.put((rank, True if not fails else repr(fails[:8])))
    except Exception as exc:  # reported to the parent
        result_q.put((rank, repr(exc)))
    finally:
        dist.destroy_process_group()


def test_two_gpu_peer_gather(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import queue
    import socket

    import torch.multiprocessing as mp

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    rq = ctx.Queue()
    procs = [ctx.Process(target=_two_rank_worker, args=(r, 2, port, rq)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = dict(rq.get(timeout=240) for _ in procs)
    except queue.Empty:
        res = {}
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.terminate()
    assert res == {0: True, 1: True}
