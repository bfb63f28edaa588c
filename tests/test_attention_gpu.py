"""Configuration-4 composition (Laplacian linear attention) against a plain
PyTorch fp64 restatement of the same formula, forward and backward."""
import math

import pytest
import torch

from laplacianformer_b200.attention import LaplacianAttention, laplacian_attention, pool_landmarks

pytestmark = pytest.mark.gpu


def reference(q, k, v, L, iters, sigma):
    def l1(a, bT):
        return (a[..., :, None, :] - bT.transpose(-1, -2)[..., None, :, :]).abs().sum(-1)

    k_ql = torch.exp(-l1(q, L.transpose(-1, -2)) / sigma)
    k_lk = torch.exp(-l1(L, k.transpose(-1, -2)) / sigma)
    A = torch.exp(-l1(L, L.transpose(-1, -2)) / sigma)
    P = A + 0.01 * torch.eye(A.shape[-1], dtype=A.dtype, device=A.device)
    alpha = 1.8 / P.sum(-1).amax(-1) ** 2
    V = P * alpha[..., None, None]
    for _ in range(iters):
        V = 2 * V - (V @ P) @ V
    return k_ql @ (V @ (k_lk @ v))


def test_block_forward_backward_fp32(cuda):
    g = torch.Generator().manual_seed(0)
    B, H, S, D = 2, 2, 8, 16
    q = torch.randn(B, H, S * S, D, generator=g, dtype=torch.float64)
    k = torch.randn(B, H, S * S, D, generator=g, dtype=torch.float64)
    v = torch.randn(B, H, S * S, D, generator=g, dtype=torch.float64)
    L = pool_landmarks(k, S, 2)
    sigma = math.sqrt(D)
    up = torch.randn(B, H, S * S, D, generator=g, dtype=torch.float64)

    qd, kd, vd = (t.float().to(cuda).requires_grad_() for t in (q, k, v))
    out = laplacian_attention(qd, kd, vd, pool_landmarks(kd, S, 2), iters=8, sigma=sigma)
    out.backward(up.float().to(cuda))

    qr, kr, vr = (t.to(cuda).requires_grad_() for t in (q, k, v))
    ref = reference(qr, kr, vr, pool_landmarks(kr, S, 2), 8, sigma)
    ref.backward(up.to(cuda))
    scale = ref.abs().max().item()
    torch.testing.assert_close(out.double(), ref.detach(), rtol=0, atol=2e-4 * scale)
    for got, want in ((qd.grad, qr.grad), (kd.grad, kr.grad), (vd.grad, vr.grad)):
        torch.testing.assert_close(got.double(), want, rtol=0, atol=2e-3 * want.abs().max().item())


def test_block_bf16_config4_shape(cuda):
    from laplacianformer_b200 import workloads

    w = workloads.config4(device=cuda, batch=4)
    q, k, v, L = (w[x].requires_grad_() if x != "landmarks" else w[x] for x in ("q", "k", "v", "landmarks"))
    out = laplacian_attention(q, k, v, L, iters=8, sigma=8.0)
    out.float().pow(2).mean().backward()
    assert out.shape == (4, 8, 196, 64) and out.dtype == torch.bfloat16
    assert torch.isfinite(out.float()).all() and torch.isfinite(q.grad.float()).all()
    ref = reference(q.detach().double(), k.detach().double(), v.detach().double(), L.double(), 8, 8.0)
    rel = (out.double() - ref).norm() / ref.norm()
    assert rel < 3e-2, rel


def test_module(cuda):
    m = LaplacianAttention(64, 4, grid=8).to(cuda)
    x = torch.randn(2, 64, 64, device=cuda, requires_grad=True)
    y = m(x)
    y.sum().backward()
    assert y.shape == x.shape and x.grad is not None


def test_landmark_inverse_autograd_matches_composition(cuda):
    """The fused landmark inverse and its backward agree with laplace_kernel
    followed by newton_inverse (same forward bits; gradients to rounding)."""
    from laplacianformer_b200.ops import landmark_inverse, laplace_kernel, newton_inverse

    g = torch.Generator().manual_seed(5)
    L = torch.randn(2, 2, 49, 64, generator=g).to(cuda)
    G = torch.randn(2, 2, 49, 49, generator=g).to(cuda)
    L1, L2 = L.clone().requires_grad_(), L.clone().requires_grad_()
    x1 = landmark_inverse(L1, -0.125, 8)
    x2 = newton_inverse(laplace_kernel(L2, L2.transpose(-1, -2).contiguous(), -0.125), 8)
    assert torch.equal(x1, x2)
    (x1 * G).sum().backward()
    (x2 * G).sum().backward()
    torch.testing.assert_close(L1.grad, L2.grad, rtol=1e-4, atol=1e-4)
