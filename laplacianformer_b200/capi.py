"""ctypes binding of the C ABI in include/laplacian_b200.h (liblfb200.so).

This is the boundary a non-Python caller binds; the tests and the end-to-end
benchmark call the kernels through it with raw device pointers, exactly as a
foreign-function caller would.  There is no fallback: if liblfb200.so is
missing the import raises.
"""
from __future__ import annotations

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liblfb200.so")

LF_F32, LF_F64, LF_F16, LF_BF16 = 0, 1, 2, 3
LF_OK, LF_ERR_INVALID, LF_ERR_DTYPE, LF_ERR_UNSUPPORTED, LF_ERR_CUDA, LF_ERR_TIMEOUT = range(6)
INIT_REFERENCE, INIT_SCALED_TRANSPOSE = 0, 1
PREC_SPLIT3, PREC_MIXED, PREC_FP32_SIMT = 0, 1, 2

_DT = {torch.float32: LF_F32, torch.float64: LF_F64, torch.float16: LF_F16, torch.bfloat16: LF_BF16}

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_D = ctypes.c_double

# name -> (restype, argtypes); the exported symbol set of include/laplacian_b200.h
SIGNATURES = {
    "lf_last_error": (ctypes.c_char_p, []),
    "lf_cudart_version": (_I, []),
    "lf_version": (_I, []),
    "lf_laplace_sub_fwd": (_I, [_P, _P, _P, _I64, _I64, _I64, _I64, _I, _P]),
    "lf_laplace_sub_fwd_packed": (_I, [_P, _P, _P, _I64, _I64, _I64, _I64, _I, _P]),
    "lf_laplace_kernel_fwd": (_I, [_P, _P, _P, _I64, _I64, _I64, _I64, _I, _D, _P]),
    "lf_laplace_kernel_bwd": (_I, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I, _D, _P, ctypes.c_size_t, _P]),
    "lf_laplace_sub_bwd_query": (_I, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I, _P]),
    "lf_laplace_sub_bwd_key": (_I, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I, _P]),
    "lf_laplace_sub_bwd": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I, _P]),
    "lf_laplace_sub_bwd_workspace_size": (ctypes.c_size_t, [_I64, _I64, _I64, _I64, _I]),
    "lf_laplace_sub_bwd_noalloc": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I, _P]),
    "lf_laplace_sub_host_buffer_size": (ctypes.c_size_t, [_I64, _I64, _I64, _I64, _I, _I]),
    "lf_laplace_sub_fwd_bwd_host": (_I, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I, _I, _P, ctypes.c_size_t,
                                         _P]),
    "lf_laplace_sub_bwd_ws": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I, _P, ctypes.c_size_t, _P]),
    "lf_laplace_sub_reduce_fwd": (_I, [_P, _P, _P, _I64, _I64, _I64, _I64, _I, _P]),
    "lf_newton_inverse_supported": (_I, [_I64]),
    "lf_newton_inverse_fwd": (_I, [_P, _P, _I64, _I64, _I, _I, _P]),
    "lf_newton_inverse_fwd_ex": (_I, [_P, _P, _I64, _I64, _I, _I, _I, _D, _I, _P]),
    "lf_laplace_newton_inverse_fwd": (_I, [_P, _P, _I64, _I64, _I64, _D, _I, _I, _D, _I, _P]),
    "lf_newton_inverse_bwd": (_I, [_P, _P, _P, _I64, _I64, _I, _P]),
    "lf_newton_inverse_residual": (_I, [_P, _P, _P, _I64, _I64, _D, _I, _P]),
    "lf_device_status": (_I, [_I]),
    "lf_selftest_bounded_wait": (_I, [_I, _P]),
    "lf_peer_alloc": (_I, [ctypes.c_size_t, ctypes.POINTER(_P), _P]),
    "lf_peer_open": (_I, [_P, ctypes.POINTER(_P)]),
    "lf_peer_close": (_I, [_P]),
    "lf_peer_free": (_I, [_P]),
    "lf_peer_put": (_I, [_P, ctypes.c_size_t, _P, _I, _P]),
    "lf_peer_barrier": (_I, [_P, _I, _I, ctypes.c_uint32, _I, _P]),
    "lf_laplace_sub_bwd_peers": (_I, [_P, _P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _I64, _I, _P, ctypes.c_size_t,
                                      _P]),
}

LF_MAX_PEERS = 8
LF_PEER_HANDLE_BYTES = 64

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m laplacianformer_b200.build` "
                "(there is no CPU fallback for these operators)"
            )
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


class LfError(RuntimeError):
    def __init__(self, code: int, where: str):
        msg = lib().lf_last_error().decode(errors="replace")
        super().__init__(f"{where} failed (code {code}): {msg}")
        self.code = code


def _check(code: int, where: str) -> None:
    if code != LF_OK:
        raise LfError(code, where)


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}") from None


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("tensors must be CUDA tensors (no CPU implementation)")
        if t is not None and not t.is_contiguous():
            raise RuntimeError("tensors must be contiguous")


def _dims(q, kT):
    B, H, N, D = q.shape
    return B * H, N, kT.shape[-1], D


def laplace_sub_fwd(q, kT, out=None):
    _need_cuda(q, kT, out)
    bh, n, m, d = _dims(q, kT)
    if out is None:
        out = torch.empty(q.shape[0], q.shape[1], n, m, device=q.device, dtype=q.dtype)
    _check(lib().lf_laplace_sub_fwd(_ptr(q), _ptr(kT), _ptr(out), bh, n, m, d, dtype_code(q), _stream(q)),
           "lf_laplace_sub_fwd")
    return out


def laplace_sub_fwd_packed(q, kT, out=None):
    """Opt-in fp16 forward in packed half2 arithmetic (within ~1e-3 relative,
    not bit-identical); fp16 tensors only, d <= 64."""
    _need_cuda(q, kT, out)
    bh, n, m, d = _dims(q, kT)
    if out is None:
        out = torch.empty(q.shape[0], q.shape[1], n, m, device=q.device, dtype=q.dtype)
    _check(lib().lf_laplace_sub_fwd_packed(_ptr(q), _ptr(kT), _ptr(out), bh, n, m, d, dtype_code(q), _stream(q)),
           "lf_laplace_sub_fwd_packed")
    return out


def laplace_kernel_fwd(q, kT, scale, out=None):
    """Kmat = exp(scale * LaplaceSub(q, kT)) in one launch (S is not stored)."""
    _need_cuda(q, kT, out)
    bh, n, m, d = _dims(q, kT)
    if out is None:
        out = torch.empty(q.shape[0], q.shape[1], n, m, device=q.device, dtype=q.dtype)
    _check(lib().lf_laplace_kernel_fwd(_ptr(q), _ptr(kT), _ptr(out), bh, n, m, d, dtype_code(q), float(scale),
                                       _stream(q)), "lf_laplace_kernel_fwd")
    return out


def laplace_kernel_bwd(gk, kmat, q, kT, scale, dq=None, dk=None, workspace=None):
    """Gradients of Kmat = exp(scale * LaplaceSub(q, kT)) from dKmat = gk, with
    dS = scale * Kmat * gk formed inside the backward kernel."""
    _need_cuda(gk, kmat, q, kT, dq, dk, workspace)
    bh, n, m, d = _dims(q, kT)
    dq = torch.empty_like(q) if dq is None else dq
    dk = torch.empty_like(kT) if dk is None else dk
    ws_ptr, ws_bytes = (None, 0) if workspace is None else (_ptr(workspace), workspace.numel() * workspace.element_size())
    _check(lib().lf_laplace_kernel_bwd(_ptr(gk), _ptr(kmat), _ptr(q), _ptr(kT), _ptr(dq), _ptr(dk), bh, n, m, d,
                                       dtype_code(q), float(scale), ws_ptr, ws_bytes, _stream(q)),
           "lf_laplace_kernel_bwd")
    return dq, dk


def laplace_sub_bwd_workspace_size(q, kT):
    """Bytes of device workspace the balanced fused backward takes for this shape (0: none)."""
    bh, n, m, d = _dims(q, kT)
    return int(lib().lf_laplace_sub_bwd_workspace_size(bh, n, m, d, dtype_code(q)))


def laplace_sub_bwd(g, q, kT, dq=True, dk=True, workspace=None):
    """Fused backward; dq/dk may be tensors, True (allocate) or None/False (skip).

    With both gradients and a shape that has a workspace size, the balanced
    kernel runs on `workspace` (a uint8 device tensor; allocated here when
    None); otherwise the workspace-free kernel runs."""
    _need_cuda(g, q, kT)
    bh, n, m, d = _dims(q, kT)
    if dq is True:
        dq = torch.empty_like(q)
    if dk is True:
        dk = torch.empty_like(kT)
    dq = dq if isinstance(dq, torch.Tensor) else None
    dk = dk if isinstance(dk, torch.Tensor) else None
    _need_cuda(dq, dk)
    need = laplace_sub_bwd_workspace_size(q, kT) if (dq is not None and dk is not None) else 0
    if need:
        if workspace is None:
            workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
        _check(lib().lf_laplace_sub_bwd_ws(_ptr(g), _ptr(q), _ptr(kT), _ptr(dq), _ptr(dk), bh, n, m, d,
                                           dtype_code(q), _ptr(workspace), workspace.numel() * workspace.element_size(),
                                           _stream(q)), "lf_laplace_sub_bwd_ws")
        return dq, dk
    _check(lib().lf_laplace_sub_bwd(_ptr(g), _ptr(q), _ptr(kT), _ptr(dq), _ptr(dk), bh, n, m, d, dtype_code(q),
                                    _stream(q)), "lf_laplace_sub_bwd")
    return dq, dk


def _ptr_table(ptrs):
    """A C array of device pointers (void* const*) kept alive by the caller."""
    return (_P * max(1, len(ptrs)))(*[int(p) for p in ptrs])


def laplace_sub_bwd_peers(g, q, kT, dq, dk, dq_peers, workspace=None):
    """laplace_sub_bwd that also stores dQ into each peer pointer of
    `dq_peers` (same layout as dq, e.g. PeerGather.peer_ptrs); both
    gradients are required."""
    _need_cuda(g, q, kT, dq, dk)
    bh, n, m, d = _dims(q, kT)
    if len(dq_peers) > LF_MAX_PEERS:
        raise ValueError(f"at most {LF_MAX_PEERS} peers")
    need = laplace_sub_bwd_workspace_size(q, kT)
    if need and workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    ws_ptr, ws_bytes = (None, 0) if workspace is None else (_ptr(workspace), workspace.numel() * workspace.element_size())
    table = _ptr_table(dq_peers)
    _check(lib().lf_laplace_sub_bwd_peers(_ptr(g), _ptr(q), _ptr(kT), _ptr(dq), _ptr(dk), table, len(dq_peers),
                                          bh, n, m, d, dtype_code(q), ws_ptr, ws_bytes, _stream(q)),
           "lf_laplace_sub_bwd_peers")
    return dq, dk


def peer_put(src, dst_ptrs, stream=None):
    """Copies the bytes of the contiguous device tensor `src` to every pointer of `dst_ptrs`."""
    _need_cuda(src)
    if not src.is_contiguous():
        raise ValueError("peer_put needs a contiguous tensor")
    st = _stream(src) if stream is None else stream.cuda_stream
    table = _ptr_table(dst_ptrs)
    _check(lib().lf_peer_put(_ptr(src), src.numel() * src.element_size(), table, len(dst_ptrs), st), "lf_peer_put")


def laplace_sub_bwd_query(g, q, kT, out=None):
    _need_cuda(g, q, kT, out)
    bh, n, m, d = _dims(q, kT)
    out = torch.empty_like(q) if out is None else out
    _check(lib().lf_laplace_sub_bwd_query(_ptr(g), _ptr(q), _ptr(kT), _ptr(out), bh, n, m, d, dtype_code(q),
                                          _stream(q)), "lf_laplace_sub_bwd_query")
    return out


def laplace_sub_bwd_key(g, q, kT, out=None):
    _need_cuda(g, q, kT, out)
    bh, n, m, d = _dims(q, kT)
    out = torch.empty_like(kT) if out is None else out
    _check(lib().lf_laplace_sub_bwd_key(_ptr(g), _ptr(q), _ptr(kT), _ptr(out), bh, n, m, d, dtype_code(q),
                                        _stream(q)), "lf_laplace_sub_bwd_key")
    return out


def laplace_sub_reduce_fwd(q, kT, out=None):
    _need_cuda(q, kT, out)
    bh, n, m, d = _dims(q, kT)
    if out is None:
        out = torch.empty(q.shape[0], q.shape[1], n, m, device=q.device, dtype=q.dtype)
    _check(lib().lf_laplace_sub_reduce_fwd(_ptr(q), _ptr(kT), _ptr(out), bh, n, m, d, dtype_code(q), _stream(q)),
           "lf_laplace_sub_reduce_fwd")
    return out


def newton_inverse_fwd(a, iters, init_mode=INIT_REFERENCE, reg=None, precision=PREC_SPLIT3, out=None):
    _need_cuda(a, out)
    n = a.shape[-1]
    batch = a.numel() // (n * n) if n else 0
    out = torch.empty_like(a) if out is None else out
    if reg is None:
        reg = 0.01 if init_mode == INIT_REFERENCE else 0.0
    _check(lib().lf_newton_inverse_fwd_ex(_ptr(a), _ptr(out), batch, n, int(iters), dtype_code(a), int(init_mode),
                                          float(reg), int(precision), _stream(a)), "lf_newton_inverse_fwd_ex")
    return out


def laplace_newton_inverse_fwd(lmk, scale, iters, init_mode=INIT_REFERENCE, reg=None, precision=PREC_SPLIT3,
                                out=None):
    """X = NewtonInverse(exp(scale * LaplaceSub(L, L^T))) in one kernel; lmk fp32 [..., n, d]."""
    _need_cuda(lmk, out)
    if lmk.dtype != torch.float32 or not lmk.is_contiguous():
        raise ValueError("landmarks must be contiguous fp32")
    n, d = lmk.shape[-2], lmk.shape[-1]
    batch = lmk.numel() // (n * d) if n * d else 0
    out = torch.empty(*lmk.shape[:-1], n, device=lmk.device, dtype=torch.float32) if out is None else out
    if reg is None:
        reg = 0.01 if init_mode == INIT_REFERENCE else 0.0
    _check(lib().lf_laplace_newton_inverse_fwd(_ptr(lmk), _ptr(out), batch, n, d, float(scale), int(iters),
                                               int(init_mode), float(reg), int(precision), _stream(lmk)),
           "lf_laplace_newton_inverse_fwd")
    return out


def newton_inverse_fwd_reference(a, iters, out=None):
    """The reference-semantics entry point lf_newton_inverse_fwd."""
    _need_cuda(a, out)
    n = a.shape[-1]
    batch = a.numel() // (n * n) if n else 0
    out = torch.empty_like(a) if out is None else out
    _check(lib().lf_newton_inverse_fwd(_ptr(a), _ptr(out), batch, n, int(iters), dtype_code(a), _stream(a)),
           "lf_newton_inverse_fwd")
    return out


def newton_inverse_bwd(g, v, out=None):
    _need_cuda(g, v, out)
    n = v.shape[-1]
    batch = v.numel() // (n * n) if n else 0
    out = torch.empty_like(v) if out is None else out
    _check(lib().lf_newton_inverse_bwd(_ptr(g), _ptr(v), _ptr(out), batch, n, dtype_code(v), _stream(v)),
           "lf_newton_inverse_bwd")
    return out


def newton_inverse_residual(a, x, reg=0.0, out=None):
    _need_cuda(a, x, out)
    n = a.shape[-1]
    batch = a.numel() // (n * n) if n else 0
    if out is None:
        out = torch.empty(batch, device=a.device, dtype=torch.float64 if a.dtype == torch.float64 else torch.float32)
    _check(lib().lf_newton_inverse_residual(_ptr(a), _ptr(x), _ptr(out), batch, n, float(reg), dtype_code(a),
                                            _stream(a)), "lf_newton_inverse_residual")
    return out


def newton_inverse_supported(n: int) -> bool:
    return bool(lib().lf_newton_inverse_supported(int(n)))


def device_status(clear: bool = True) -> int:
    return int(lib().lf_device_status(1 if clear else 0))
