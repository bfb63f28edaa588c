"""PyTorch autograd front end for the B200 operators.

The reference ships the two operators as raw out-parameter functions with no
``autograd.Function`` (it only exposes ``Laplace_subtraction_cuda``); the
paper's attention module calls forward and the two backward ops itself.
These wrappers give that composition:

* :func:`laplace_subtraction` — ``S = LaplaceSub(Q, K^T)``; backward runs the
  fused one-pass kernel for dQ and dK^T.
* :func:`newton_inverse` — Newton–Schulz inverse; backward is the reference's
  analytic ``-V^T G V^T`` (src/NewtonInverse_cuda_kernel.cu:466-573).

Every call goes to the ``Laplace_subtraction_cuda`` extension; there is no CPU
fallback and a missing extension raises ImportError.
"""
from __future__ import annotations

import torch

_EXT = None


def ext():
    """The compiled Laplace_subtraction_cuda module (raises if it is missing)."""
    global _EXT
    if _EXT is None:
        try:
            import Laplace_subtraction_cuda as m  # noqa: N813
        except ImportError as e:  # pragma: no cover - depends on the build
            raise ImportError(
                "Laplace_subtraction_cuda is not built; run `python setup.py build_ext --inplace` "
                "(there is no CPU fallback for these operators)"
            ) from e
        _EXT = m
    return _EXT


INIT_REFERENCE, INIT_SCALED_TRANSPOSE = 0, 1
PREC_SPLIT3, PREC_MIXED, PREC_FP32_SIMT = 0, 1, 2


class LaplaceSubtractionFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, query, key):
        query = query.contiguous()
        key = key.contiguous()
        out = query.new_empty(query.shape[0], query.shape[1], query.shape[2], key.shape[3])
        ext().LaplaceSubtraction_forward(query, key, out)
        ctx.save_for_backward(query, key)
        return out

    @staticmethod
    def backward(ctx, grad):
        query, key = ctx.saved_tensors
        need_q, need_k = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        dq = torch.empty_like(query) if need_q else None
        dk = torch.empty_like(key) if need_k else None
        if need_q or need_k:
            ext().LaplaceSubtraction_backward(grad.contiguous(), query, key, dq, dk)
        return dq, dk


def laplace_subtraction(query: torch.Tensor, key: torch.Tensor) -> torch.Tensor:
    """S[b,h,n,m] = sum_d |query[b,h,n,d] - key[b,h,d,m]| with key given as [B,H,D,M]."""
    return LaplaceSubtractionFn.apply(query, key)


class LaplaceKernelFn(torch.autograd.Function):
    """Kmat = exp(scale * LaplaceSub(Q, K^T)), forward fused into one kernel;
    backward in one kernel too: dS = scale * Kmat * dKmat is formed while the
    fused LaplaceSub backward stages its gradient tile (LaplaceKernel_backward)."""

    @staticmethod
    def forward(ctx, query, key, scale):
        query = query.contiguous()
        key = key.contiguous()
        out = query.new_empty(query.shape[0], query.shape[1], query.shape[2], key.shape[3])
        ext().LaplaceKernel_forward(query, key, out, float(scale))
        ctx.save_for_backward(query, key, out)
        ctx.scale = float(scale)
        return out

    @staticmethod
    def backward(ctx, grad):
        query, key, out = ctx.saved_tensors
        need_q, need_k = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        dq = torch.empty_like(query) if need_q else None
        dk = torch.empty_like(key) if need_k else None
        if need_q or need_k:
            ext().LaplaceKernel_backward(grad.contiguous(), out, ctx.scale, query, key, dq, dk)
        return dq, dk, None


def laplace_kernel(query: torch.Tensor, key: torch.Tensor, scale: float) -> torch.Tensor:
    """exp(scale * sum_d |query - key|) with key given as [B,H,D,M]; S is never materialised."""
    return LaplaceKernelFn.apply(query, key, scale)


class NewtonInverseFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, mat, iters, init_mode, reg, precision):
        mat = mat.contiguous()
        out = torch.empty_like(mat)
        ext().NewtonInverse_forward_ex(mat, out, int(iters), int(init_mode), float(reg), int(precision))
        ctx.save_for_backward(out)
        return out

    @staticmethod
    def backward(ctx, grad):
        (inv,) = ctx.saved_tensors
        dmat = torch.empty_like(inv)
        ext().NewtonInverse_backward(grad.contiguous(), inv, dmat)
        return dmat, None, None, None, None


def newton_inverse(mat: torch.Tensor, iters: int, init_mode: int = INIT_REFERENCE, reg: float | None = None,
                   precision: int = PREC_SPLIT3) -> torch.Tensor:
    """Newton–Schulz inverse of [B,H,N,N] matrices (reference semantics by default)."""
    if reg is None:
        reg = 0.01 if init_mode == INIT_REFERENCE else 0.0
    return NewtonInverseFn.apply(mat, iters, init_mode, reg, precision)


class LandmarkInverseFn(torch.autograd.Function):
    """X = NewtonInverse(exp(scale * LaplaceSub(L, L^T))) with A built inside
    the inverse kernel (lf_laplace_newton_inverse_fwd).  Backward:
    dA = -X^T G X^T (the inverse's analytic backward), dS = scale * A * dA with
    A recomputed by the fused exp forward, then the LaplaceKernel backward
    (dS formed inside it) with L as both query and key: dL = dQ + (dK^T)^T."""

    @staticmethod
    def forward(ctx, lmk, scale, iters, init_mode, reg, precision):
        from . import capi

        lmk = lmk.contiguous()
        x = capi.laplace_newton_inverse_fwd(lmk, scale, iters, init_mode=init_mode, reg=reg, precision=precision)
        ctx.save_for_backward(lmk, x)
        ctx.scale = float(scale)
        return x

    @staticmethod
    def backward(ctx, grad):
        lmk, x = ctx.saved_tensors
        da = torch.empty_like(x)
        ext().NewtonInverse_backward(grad.contiguous(), x, da)
        lT = lmk.transpose(-1, -2).contiguous()
        a = torch.empty_like(x)
        ext().LaplaceKernel_forward(lmk, lT, a, ctx.scale)
        dq = torch.empty_like(lmk)
        dkT = torch.empty_like(lT)
        ext().LaplaceKernel_backward(da, a, ctx.scale, lmk, lT, dq, dkT)  # dS = scale * A * dA in the kernel
        return dq + dkT.transpose(-1, -2), None, None, None, None, None


def landmark_inverse(lmk: torch.Tensor, scale: float, iters: int, init_mode: int = INIT_REFERENCE,
                     reg: float | None = None, precision: int = PREC_SPLIT3) -> torch.Tensor:
    """Inverse of the landmark kernel matrix exp(scale * cdist_1(L, L)) for fp32 L [B,H,M,D], M <= 128,
    D <= 128, in one kernel (the matrix is never stored)."""
    if reg is None:
        reg = 0.01 if init_mode == INIT_REFERENCE else 0.0
    return LandmarkInverseFn.apply(lmk, scale, iters, init_mode, reg, precision)


def newton_residual(mat: torch.Tensor, inv: torch.Tensor, reg: float = 0.0) -> torch.Tensor:
    """||(A + reg I) X - I||_F per matrix, shape [B,H]."""
    res = torch.empty(mat.shape[0], mat.shape[1], device=mat.device,
                      dtype=torch.float64 if mat.dtype == torch.float64 else torch.float32)
    ext().NewtonInverse_residual(mat.contiguous(), inv.contiguous(), res, float(reg))
    return res
