"""Generate golden vectors by running the REFERENCE operators.

Run on a machine with a CUDA GPU after `python oracle/build_ref.py` has
compiled the reference sources into oracle/_ref/:

    python tests/golden/make_golden.py [OUT_DIR]

Each laplace_*.npz holds seeded inputs (q [B,H,N,D], k [B,H,D,M], g [B,H,N,M])
and the reference's outputs of LaplaceSubtraction_forward, _backward_query,
_backward_key and _reduce_forward; each newton_*.npz holds SPD kernel
matrices A, the reference's NewtonInverse_forward output X for `iters`
iterations, an upstream gradient G and NewtonInverse_backward's dA.
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle.build_ref import load_ref  # noqa: E402

LAPLACE_CASES = [
    # name, B, H, N, D, M, dtype
    ("f32_vit", 2, 2, 70, 32, 49, torch.float32),
    ("f32_ragged", 1, 3, 33, 17, 5, torch.float32),
    ("f32_d48", 1, 1, 20, 48, 9, torch.float32),
    ("f32_m64", 1, 2, 64, 64, 64, torch.float32),
    ("f64_small", 1, 2, 20, 9, 7, torch.float64),
    ("f16_vit", 2, 2, 70, 32, 49, torch.float16),
]
NEWTON_CASES = [
    # name, batch, n, iters
    ("f32_n64", 4, 64, 10),
    ("f32_n128", 4, 128, 12),
    ("f32_n49", 3, 49, 8),
    ("f32_n100", 2, 100, 12),
]


def spd(batch, n, seed, d=16, sigma=4.0):
    g = torch.Generator().manual_seed(seed)
    L = torch.randn(batch, n, d, generator=g, dtype=torch.float64)
    return (torch.exp(-torch.cdist(L, L, p=1) / sigma) + 1e-3 * torch.eye(n, dtype=torch.float64)).float()


def main(out_dir):
    ref = load_ref()
    assert ref is not None, "build the reference first: python oracle/build_ref.py"
    dev = torch.device("cuda:0")
    for i, (name, B, H, N, D, M, dt) in enumerate(LAPLACE_CASES):
        g = torch.Generator().manual_seed(100 + i)
        q = torch.randn(B, H, N, D, generator=g).to(dt)
        k = torch.randn(B, H, D, M, generator=g).to(dt)
        gr = torch.randn(B, H, N, M, generator=g).to(dt)
        qd, kd, gd = q.to(dev), k.to(dev), gr.to(dev)
        s = torch.empty(B, H, N, M, device=dev, dtype=dt)
        ref.LaplaceSubtraction_forward(qd, kd, s)
        dq = torch.empty_like(qd)
        ref.LaplaceSubtraction_backward_query(gd, qd, kd, dq)
        dk = torch.empty_like(kd)
        ref.LaplaceSubtraction_backward_key(gd, qd, kd, dk)
        r = torch.empty_like(s)
        ref.LaplaceSubtraction_reduce_forward(qd, kd, r)
        torch.cuda.synchronize()
        wide = torch.float64 if dt == torch.float64 else torch.float32
        np.savez_compressed(
            os.path.join(out_dir, f"laplace_{name}.npz"),
            q=q.to(wide).numpy(), k=k.to(wide).numpy(), g=gr.to(wide).numpy(),
            s=s.cpu().to(wide).numpy(), dq=dq.cpu().to(wide).numpy(), dk=dk.cpu().to(wide).numpy(),
            reduce=r.cpu().to(wide).numpy(), dtype=str(dt).replace("torch.", ""),
        )
    for i, (name, batch, n, iters) in enumerate(NEWTON_CASES):
        A = spd(batch, n, 200 + i).view(1, batch, n, n)
        G = torch.randn(1, batch, n, n, generator=torch.Generator().manual_seed(300 + i))
        Ad, Gd = A.to(dev), G.to(dev)
        X = torch.empty_like(Ad)
        ref.NewtonInverse_forward(Ad, X, iters)
        dA = torch.empty_like(Ad)
        ref.NewtonInverse_backward(Gd, X, dA)
        torch.cuda.synchronize()
        np.savez_compressed(
            os.path.join(out_dir, f"newton_{name}.npz"),
            A=A.numpy(), X=X.cpu().numpy(), G=G.numpy(), dA=dA.cpu().numpy(), iters=iters,
        )
    print("wrote goldens to", out_dir)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else HERE)
