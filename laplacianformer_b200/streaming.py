"""LaplaceSubtraction forward + both gradients for host-resident batches.

When Q, K^T and dS live in (pinned) host memory, the PCIe copies dominate:
a configuration-2 step moves 65 MB in and 65 MB out against ~0.15 ms of
kernels.  :class:`HostPipeline` drives ``lf_laplace_sub_fwd_bwd_host``: the
B*H slices are split into chunks that flow through three CUDA streams —
host-to-device copies, the two kernels, device-to-host copies — over a ring
of three device buffer sets, so the copy-in of chunk i+1, the kernels of
chunk i and the copy-out of chunk i-1 overlap (PCIe is full duplex).  The
chunk loop runs in the library (C++), so enqueueing costs a few microseconds
per chunk.  The device buffer is allocated once per pipeline.
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
        code = capi.dtype_code(torch.empty(0, dtype=dtype))
        self.code = code
        with torch.cuda.device(self.device):
            need = int(capi.lib().lf_laplace_sub_host_buffer_size(self.bh, N, m, D, code, self.chunks))
        # 256-byte aligned (the caching allocator aligns to 512)
        self.dbuf = torch.empty(need, dtype=torch.uint8, device=self.device)

    def __call__(self, q, kT, ds, s, dq, dkT):
        for t in (q, kT, ds, s, dq, dkT):
            if t.device.type != "cpu" or t.dtype != self.dtype or not t.is_contiguous():
                raise ValueError("HostPipeline takes contiguous host tensors of the pipeline's dtype")
        L = capi.lib()
        with torch.cuda.device(self.device):
            st = torch.cuda.current_stream(self.device)
            rc = L.lf_laplace_sub_fwd_bwd_host(q.data_ptr(), kT.data_ptr(), ds.data_ptr(), s.data_ptr(),
                                               dq.data_ptr(), dkT.data_ptr(), self.bh, self.n, self.m, self.d,
                                               self.code, self.chunks, self.dbuf.data_ptr(), self.dbuf.numel(),
                                               st.cuda_stream)
        capi._check(rc, "lf_laplace_sub_fwd_bwd_host")
        return s, dq, dkT
