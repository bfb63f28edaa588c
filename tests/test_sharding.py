"""B*H sharding logic on CPU: split arithmetic, and world_size-2 gloo ranks
computing their slices with the CPU oracle and all-gathering them — the same
code path multi-GPU callers use with NCCL.  Also a rank that leaves before the
collective: the survivor gets an error, not a hang."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from laplacianformer_b200.sharding import all_gather_bh, flatten_bh, local_slice, run_sharded, shard_bounds


@pytest.mark.parametrize("total,world", [(128, 8), (64, 2), (10, 4), (3, 4), (0, 2), (7, 1)])
def test_bounds_partition(total, world):
    spans = [shard_bounds(total, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == total
    for (s0, e0), (s1, e1) in zip(spans, spans[1:]):
        assert e0 == s1
    sizes = [e - s for s, e in spans]
    assert max(sizes) - min(sizes) <= 1


def test_local_slice_is_contiguous_view():
    t = torch.arange(2 * 3 * 4).view(2, 3, 4)
    sl = local_slice(t, 4, 1)
    s, e = shard_bounds(6, 4, 1)
    assert torch.equal(sl, flatten_bh(t)[s:e])
    assert sl.data_ptr() == flatten_bh(t)[s].data_ptr()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, **kw):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, **kw)


def _worker(rank, world, port, bh, result_q):
    _init(rank, world, port)
    try:
        from oracle import oracle as O

        g = torch.Generator().manual_seed(0)
        q = torch.randn(bh // 2, 2, 40, 8, generator=g)
        k = torch.randn(bh // 2, 2, 8, 5, generator=g)
        up = torch.randn(bh // 2, 2, 40, 5, generator=g)

        def fn(ql, kl, gl):
            s = torch.from_numpy(O.laplace_fwd(ql.numpy(), kl.numpy()))
            dq = torch.from_numpy(O.laplace_bwd_query(gl.numpy(), ql.numpy(), kl.numpy()))
            dk = torch.from_numpy(O.laplace_bwd_key(gl.numpy(), ql.numpy(), kl.numpy()))
            return s, dq, dk

        outs = run_sharded(fn, [q, k, up])
        full = fn(q.reshape(1, bh, 40, 8), k.reshape(1, bh, 8, 5), up.reshape(1, bh, 40, 5))
        ok = all(torch.equal(a, flatten_bh(b)) for a, b in zip(outs, full))
        A = torch.eye(6).repeat(bh // 2, 2, 1, 1) * 2.0
        (X,) = run_sharded(lambda a: (torch.from_numpy(O.newton_fwd(a.numpy(), 20)),), [A])
        inv = np.linalg.inv(A.reshape(bh, 6, 6).numpy() + 0.01 * np.eye(6))
        ok = ok and X.shape == (bh, 6, 6) and np.allclose(X.numpy(), inv, atol=1e-5)
        result_q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


def _spawn(target, extra=()):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, 2, port, *extra, q)) for r in range(2)]
    for p in procs:
        p.start()
    return q, procs


def _run_pair(target, extra=(), timeout=120):
    """Run two gloo ranks and collect {rank: result}.  A rendezvous on a port
    that another process grabbed between _free_port and the bind can hang;
    such an attempt is terminated and retried once on a fresh port."""
    import queue as _queue

    for attempt in range(2):
        q, procs = _spawn(target, extra)
        try:
            res = dict(q.get(timeout=timeout) for _ in procs)
        except _queue.Empty:
            for p in procs:
                p.terminate()
                p.join(timeout=10)
            if attempt == 1:
                raise
            continue
        for p in procs:
            p.join(timeout=60)
        return res


@pytest.mark.parametrize("bh", [8, 6])
def test_two_gloo_ranks_match_single_process(bh):
    res = _run_pair(_worker, (bh,))
    assert res == {0: True, 1: True}


def _gather_uneven(rank, world, port, result_q):
    _init(rank, world, port)
    try:
        s, e = shard_bounds(5, world, rank)
        local = torch.arange(s, e, dtype=torch.float32).view(-1, 1).repeat(1, 3)
        out = all_gather_bh(local, 5)
        result_q.put((rank, torch.equal(out[:, 0], torch.arange(5, dtype=torch.float32))))
    finally:
        dist.destroy_process_group()


def test_uneven_all_gather():
    res = _run_pair(_gather_uneven)
    assert res == {0: True, 1: True}


def _leaver(rank, world, port, result_q):
    import datetime

    _init(rank, world, port, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # leaves between steps, before the collective
    try:
        all_gather_bh(torch.zeros(1, 2), 2)
        result_q.put((rank, "no error"))
    except Exception:
        result_q.put((rank, "error"))
    finally:
        os._exit(0)


def _overlap_worker(rank, world, port, bh, chunks, result_q):
    _init(rank, world, port)
    try:
        from laplacianformer_b200.sharding import run_sharded_overlapped

        g = torch.Generator().manual_seed(1)
        q = torch.randn(1, bh, 12, 4, generator=g)
        k = torch.randn(1, bh, 4, 3, generator=g)

        def fn(ql, kl):
            d = (ql.unsqueeze(-1) - kl.unsqueeze(-3)).abs().sum(-2)  # [1, b, 12, 3]
            return d, ql * 2.0

        ref = run_sharded(fn, [q, k])
        got = run_sharded_overlapped(fn, [q, k], chunks=chunks)
        ok = all(torch.equal(a, b) for a, b in zip(ref, got)) and got[0].shape[0] == bh
        result_q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("bh,chunks", [(8, 3), (7, 2), (3, 4), (5, 1)])
def test_overlapped_gather_matches_run_sharded(bh, chunks):
    res = _run_pair(_overlap_worker, (bh, chunks))
    assert res == {0: True, 1: True}


def test_rank_leaving_before_collective_raises():
    q, procs = _spawn(_leaver)
    rank, what = q.get(timeout=180)
    for p in procs:
        p.join(timeout=60)
    assert rank == 0 and what == "error"
