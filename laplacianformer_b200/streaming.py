"""LaplaceSubtraction forward + both gradients for host-resident batches.

When Q, K^T and dS live in (pinned) host memory, the PCIe copies dominate:
a configuration-2 step moves 65 MB in and 65 MB out against ~0.2 ms of
kernels.  :class:`HostPipeline` splits the B*H slices into chunks and runs
three CUDA streams — host-to-device copies, the two kernels, device-to-host
copies — so that the copy-in of chunk i+1, the kernels of chunk i and the
copy-out of chunk i-1 overlap (PCIe is full duplex).  Device buffers are
allocated once per pipeline (double-buffered per chunk); each call only
enqueues work and returns after the last copy-out completed.
"""
from __future__ import annotations

import torch

from . import capi


class HostPipeline:
    """Streams fwd+bwd over B*H chunks of pinned host tensors.

    q [B,H,N,D], kT [B,H,D,M], ds [B,H,N,M] -> s [B,H,N,M], dq [B,H,N,D],
    dkT [B,H,D,M], all pinned host tensors of one dtype.
    """

    def __init__(self, shape_q, m: int, dtype=torch.float32, device=None, chunks: int = 8):
        B, H, N, D = shape_q
        self.bh, self.n, self.d, self.m = B * H, N, D, m
        self.dtype = dtype
        self.device = torch.device(device if device is not None else "cuda")
        self.chunks = max(1, min(chunks, self.bh))
        self.per = -(-self.bh // self.chunks)
        dev, per = self.device, self.per
        # two buffer sets: chunk i uses set i % 2
        self.buf = [
            {
                "q": torch.empty(per, N, D, device=dev, dtype=dtype),
                "k": torch.empty(per, D, m, device=dev, dtype=dtype),
                "g": torch.empty(per, N, m, device=dev, dtype=dtype),
                "s": torch.empty(per, N, m, device=dev, dtype=dtype),
                "dq": torch.empty(per, N, D, device=dev, dtype=dtype),
                "dk": torch.empty(per, D, m, device=dev, dtype=dtype),
            }
            for _ in range(2)
        ]
        self.s_in = torch.cuda.Stream(dev)
        self.s_run = torch.cuda.Stream(dev)
        self.s_out = torch.cuda.Stream(dev)

    def __call__(self, q, kT, ds, s, dq, dkT):
        bh, per = self.bh, self.per
        qf, kf, gf = q.view(bh, self.n, self.d), kT.view(bh, self.d, self.m), ds.view(bh, self.n, self.m)
        sf, dqf, dkf = s.view(bh, self.n, self.m), dq.view(bh, self.n, self.d), dkT.view(bh, self.d, self.m)
        start = torch.cuda.current_stream(self.device)
        ev_start = torch.cuda.Event()
        ev_start.record(start)
        loaded, done, freed = [], [], []
        nchunks = -(-bh // per)
        for i in range(nchunks):
            a, b = i * per, min(bh, (i + 1) * per)
            w = b - a
            bufs = self.buf[i % 2]
            # copy-in (waits until the copy-out two chunks back released this buffer set)
            self.s_in.wait_event(ev_start)
            if i >= 2:
                self.s_in.wait_event(freed[i - 2])
            with torch.cuda.stream(self.s_in):
                bufs["q"][:w].copy_(qf[a:b], non_blocking=True)
                bufs["k"][:w].copy_(kf[a:b], non_blocking=True)
                bufs["g"][:w].copy_(gf[a:b], non_blocking=True)
                e = torch.cuda.Event()
                e.record(self.s_in)
                loaded.append(e)
            # kernels
            self.s_run.wait_event(loaded[i])
            with torch.cuda.stream(self.s_run):
                qv = bufs["q"][:w].unsqueeze(0)
                kv = bufs["k"][:w].unsqueeze(0)
                gv = bufs["g"][:w].unsqueeze(0)
                capi.laplace_sub_fwd(qv, kv, bufs["s"][:w].unsqueeze(0))
                capi.laplace_sub_bwd(gv, qv, kv, bufs["dq"][:w].unsqueeze(0), bufs["dk"][:w].unsqueeze(0))
                e = torch.cuda.Event()
                e.record(self.s_run)
                done.append(e)
            # copy-out
            self.s_out.wait_event(done[i])
            with torch.cuda.stream(self.s_out):
                sf[a:b].copy_(bufs["s"][:w], non_blocking=True)
                dqf[a:b].copy_(bufs["dq"][:w], non_blocking=True)
                dkf[a:b].copy_(bufs["dk"][:w], non_blocking=True)
                e = torch.cuda.Event()
                e.record(self.s_out)
                freed.append(e)
        start.wait_event(freed[-1])
        return s, dq, dkT
