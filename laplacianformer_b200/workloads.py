"""Seeded synthetic inputs with the shapes of the benchmark configurations.

No dataset is involved: every configuration draws N(0,1) tensors from a
seeded generator in a fixed order (query, key or key grid, upstream
gradient), builds landmarks the way the configuration describes, and passes
them to the operators in the reference layout (key transposed, [B,H,D,M]).
"""
from __future__ import annotations

import math

import torch


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _randn(shape, g, device, dtype=torch.float32):
    return torch.randn(*shape, generator=g, device=device, dtype=torch.float32).to(dtype)


def chunk_mean_landmarks(k: torch.Tensor, m: int) -> torch.Tensor:
    """[B,H,N,D] -> [B,H,M,D]: mean over M contiguous chunks of N/M tokens."""
    B, H, N, D = k.shape
    return k.view(B, H, m, N // m, D).float().mean(3).to(k.dtype)


def pooled_landmarks(grid: torch.Tensor, pool: int) -> torch.Tensor:
    """[B,H,S,S,D] key grid -> [B,H,(S/pool)^2,D] by pool x pool average pooling."""
    B, H, S, S2, D = grid.shape
    s = S // pool
    g = grid.float().view(B, H, s, pool, s, pool, D).mean((3, 5))
    return g.reshape(B, H, s * s, D).to(grid.dtype)


def kernel_matrix(landmarks: torch.Tensor, sigma: float) -> torch.Tensor:
    """A = exp(-cdist_1(L, L) / sigma) for landmarks [..., M, D] (fp32 math)."""
    L = landmarks.float()
    S = torch.cdist(L, L, p=1)
    return torch.exp(-S / sigma)


def config1(device="cpu", seed=0):
    """CPU-runnable check: Q,K [1,1,1024,32]; 64 chunk-mean landmarks; sigma = sqrt(32)."""
    g = _gen(seed, device)
    q = _randn((1, 1, 1024, 32), g, device)
    k = _randn((1, 1, 1024, 32), g, device)
    L = chunk_mean_landmarks(k, 64)
    kT = L.transpose(-1, -2).contiguous()
    A = kernel_matrix(L, math.sqrt(32.0))
    return {"q": q, "k": k, "landmarks": L, "kT": kT, "A": A, "iters": 10, "sigma": math.sqrt(32.0)}


def config2(device="cpu", dtype=torch.float32, seed=0, batch=32):
    """Pyramid-ViT stage 1: Q [B,2,3136,32]; 49 landmarks from 8x8 pooling of a
    56x56 N(0,1) key grid; upstream gradient dS [B,2,3136,49] N(0,1)."""
    g = _gen(seed, device)
    q = _randn((batch, 2, 3136, 32), g, device, dtype)
    grid = _randn((batch, 2, 56, 56, 32), g, device)
    L = pooled_landmarks(grid, 8).to(dtype)
    kT = L.transpose(-1, -2).contiguous()
    ds = _randn((batch, 2, 3136, 49), g, device, dtype)
    return {"q": q, "kT": kT, "ds": ds}


def config3(device="cpu", seed=0, batch=4096, n=128, d=64, sigma=8.0):
    """Batched inverse: A = exp(-cdist_1(L,L)/sigma) + 1e-3 I, L ~ N(0,1) [n,d]
    per matrix; returned as [batch/64, 64, n, n] (or [1,batch,n,n])."""
    g = _gen(seed, device)
    L = _randn((batch, n, d), g, device)
    A = kernel_matrix(L, sigma) + 1e-3 * torch.eye(n, device=device)
    h = 64 if batch % 64 == 0 else batch
    return {"A": A.view(batch // h, h, n, n).contiguous(), "iters": 12}


def config4(device="cpu", seed=0, batch=128):
    """14x14 ViT stage: Q,K,V [B,8,196,64] bf16, 49 landmarks from 2x2 pooling
    of K on the 14x14 grid, sigma = sqrt(64) (assumed; the config does not state it)."""
    g = _gen(seed, device)
    q = _randn((batch, 8, 196, 64), g, device, torch.bfloat16)
    k = _randn((batch, 8, 196, 64), g, device, torch.bfloat16)
    v = _randn((batch, 8, 196, 64), g, device, torch.bfloat16)
    L = pooled_landmarks(k.view(batch, 8, 14, 14, 64), 2)
    return {"q": q, "k": k, "v": v, "landmarks": L, "iters": 8, "sigma": 8.0}


def config5(n_tokens, device="cpu", seed=0, heads=16, batch=8, d=64, m=256):
    """Long sequence: Q,K [8,16,N,64] bf16, 256 chunk-mean landmarks."""
    g = _gen(seed, device)
    q = _randn((batch, heads, n_tokens, d), g, device, torch.bfloat16)
    k = _randn((batch, heads, n_tokens, d), g, device, torch.bfloat16)
    L = chunk_mean_landmarks(k, m)
    return {"q": q, "k": k, "landmarks": L, "kT": L.transpose(-1, -2).contiguous(), "iters": 10}
