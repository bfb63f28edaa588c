"""CPU oracle for the LaplacianFormer operators — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` (as the checker) and ``bench.py``
(the timed CPU baseline and the reference arm) may import this module.  The
product package never imports it.

The arithmetic lives in ``oracle/oracle.c`` (a plain-C restatement of the
reference kernels, each routine citing the reference file:line it follows);
this module loads it with ctypes, splits the outermost index over host threads
(ctypes releases the GIL during the call) and handles dtype conversion the
way the reference does:

* fp32 / fp64 inputs are computed in their own type;
* fp16 / bf16 inputs are widened to fp32, computed in fp32 and rounded back
  (``AccT<half> = float``, LaplaceSubtraction_cuda_kernel.cu:17-29 and
  NewtonInverse_cuda_kernel.cu:17-29);
* the legacy reduce forward accumulates in the storage type
  (LaplaceSubtraction_cuda_kernel.cu:429-433), restated with ``_Float16``.

Tensor layouts are the reference's: Q ``[B,H,N,D]``, key ``[B,H,D,M]``
(transposed landmarks), S and dS ``[B,H,N,M]``; matrices ``[B,H,N,N]``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from concurrent.futures import ThreadPoolExecutor

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None
_lock = threading.Lock()

_P = ctypes.c_void_p
_I64 = ctypes.c_int64


def build(force: bool = False) -> str:
    """Compile oracle.c into oracle/liboracle.so (gcc, seconds)."""
    if force or not os.path.exists(_LIB_PATH) or (
        os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "oracle.c"))
    ):
        subprocess.check_call(["make", "-s", "-C", _HERE, "-B" if force else "liboracle.so"])
    return _LIB_PATH


def lib():
    global _lib
    with _lock:
        if _lib is None:
            build()
            L = ctypes.CDLL(_LIB_PATH)
            for name in ("fwd", "bwd_query", "bwd_key", "reduce"):
                for t in ("f32", "f64") + (("f16",) if name == "reduce" else ()):
                    fn = getattr(L, f"lfo_laplace_{name}_{t}")
                    fn.restype = None
                    if name in ("fwd", "reduce"):
                        fn.argtypes = [_P, _P, _P, _I64, _I64, _I64, _I64]
                    else:
                        fn.argtypes = [_P, _P, _P, _P, _I64, _I64, _I64, _I64]
            for t, ct in (("f32", ctypes.c_float), ("f64", ctypes.c_double)):
                fn = getattr(L, f"lfo_newton_fwd_{t}")
                fn.restype = None
                fn.argtypes = [_P, _P, _I64, _I64, ctypes.c_int, ctypes.c_int, ct, ctypes.c_int]
                fn = getattr(L, f"lfo_newton_bwd_{t}")
                fn.restype = None
                fn.argtypes = [_P, _P, _P, _I64, _I64]
            _lib = L
    return _lib


_threads = max(1, os.cpu_count() or 1)


def set_threads(n: int) -> None:
    global _threads
    _threads = max(1, int(n))


def threads() -> int:
    return _threads


def _chunks(total: int):
    k = max(1, min(_threads, total))
    step = (total + k - 1) // k
    return [(s, min(total, s + step)) for s in range(0, total, step)]


def _run(jobs):
    if len(jobs) == 1:
        jobs[0]()
        return
    with ThreadPoolExecutor(max_workers=len(jobs)) as ex:
        list(ex.map(lambda f: f(), jobs))


def _ptr(a: np.ndarray, off_elems: int = 0) -> int:
    return a.ctypes.data + off_elems * a.itemsize


def _compute_dtype(dt):
    dt = np.dtype(dt)
    if dt == np.float64:
        return np.float64, "f64"
    return np.float32, "f32"


def _np(x):
    """Accept numpy arrays or torch tensors (bf16 tensors are widened)."""
    if hasattr(x, "detach"):
        import torch

        t = x.detach().cpu()
        if t.dtype == torch.bfloat16:
            return t.float().numpy(), "bfloat16"
        return t.numpy(), str(t.dtype).replace("torch.", "")
    x = np.asarray(x)
    return x, str(x.dtype)


def _round_to(x: np.ndarray, name: str):
    if name == "float16":
        return x.astype(np.float16)
    if name == "bfloat16":
        import torch

        return torch.from_numpy(np.ascontiguousarray(x)).to(torch.bfloat16)
    if name == "float32":
        return x.astype(np.float32)
    return x


def _dims(q, k):
    assert q.ndim == 4 and k.ndim == 4, "4D tensors expected"
    B, H, N, D = q.shape
    assert k.shape[0] == B and k.shape[1] == H and k.shape[2] == D, "query and key must match"
    return B, H, N, k.shape[3], D


# --------------------------------------------------------------------------
# LaplaceSubtraction
# --------------------------------------------------------------------------
def laplace_fwd(query, key):
    """S[b,h,n,m] = sum_d |Q[b,h,n,d] - K[b,h,d,m]| (LaplaceSubtraction_cuda_kernel.cu:47-141)."""
    qn, name = _np(query)
    kn, _ = _np(key)
    B, H, N, M, D = _dims(qn, kn)
    ct, tag = _compute_dtype(qn.dtype)
    q = np.ascontiguousarray(qn, dtype=ct)
    k = np.ascontiguousarray(kn, dtype=ct)
    s = np.empty((B, H, N, M), dtype=ct)
    fn = getattr(lib(), f"lfo_laplace_fwd_{tag}")
    BH = B * H
    jobs = [
        (lambda a=a, b=b: fn(_ptr(q, a * N * D), _ptr(k, a * D * M), _ptr(s, a * N * M), b - a, N, M, D))
        for a, b in _chunks(BH)
    ] if BH > 1 else [
        (lambda a=a, b=b: fn(_ptr(q, a * D), _ptr(k), _ptr(s, a * M), 1, b - a, M, D)) for a, b in _chunks(N)
    ]
    _run(jobs)
    return _round_to(s, name)


def laplace_bwd_query(grad, query, key):
    """dQ = sum_m dS * sign(Q - K) (LaplaceSubtraction_cuda_kernel.cu:148-267)."""
    gn, _ = _np(grad)
    qn, name = _np(query)
    kn, _ = _np(key)
    B, H, N, M, D = _dims(qn, kn)
    ct, tag = _compute_dtype(qn.dtype)
    g = np.ascontiguousarray(gn, dtype=ct)
    q = np.ascontiguousarray(qn, dtype=ct)
    k = np.ascontiguousarray(kn, dtype=ct)
    dq = np.empty((B, H, N, D), dtype=ct)
    fn = getattr(lib(), f"lfo_laplace_bwd_query_{tag}")
    BH = B * H
    if BH > 1:
        jobs = [
            (lambda a=a, b=b: fn(_ptr(g, a * N * M), _ptr(q, a * N * D), _ptr(k, a * D * M), _ptr(dq, a * N * D), b - a, N, M, D))
            for a, b in _chunks(BH)
        ]
    else:
        jobs = [
            (lambda a=a, b=b: fn(_ptr(g, a * M), _ptr(q, a * D), _ptr(k), _ptr(dq, a * D), 1, b - a, M, D))
            for a, b in _chunks(N)
        ]
    _run(jobs)
    return _round_to(dq, name)


def laplace_bwd_key(grad, query, key):
    """dK = -sum_n dS * sign(Q - K) (LaplaceSubtraction_cuda_kernel.cu:274-393)."""
    gn, _ = _np(grad)
    qn, name = _np(query)
    kn, _ = _np(key)
    B, H, N, M, D = _dims(qn, kn)
    ct, tag = _compute_dtype(qn.dtype)
    g = np.ascontiguousarray(gn, dtype=ct)
    q = np.ascontiguousarray(qn, dtype=ct)
    k = np.ascontiguousarray(kn, dtype=ct)
    dk = np.empty((B, H, D, M), dtype=ct)
    fn = getattr(lib(), f"lfo_laplace_bwd_key_{tag}")
    jobs = [
        (lambda a=a, b=b: fn(_ptr(g, a * N * M), _ptr(q, a * N * D), _ptr(k, a * D * M), _ptr(dk, a * D * M), b - a, N, M, D))
        for a, b in _chunks(B * H)
    ]
    _run(jobs)
    return _round_to(dk, name)


def laplace_reduce(query, key):
    """Legacy reduce forward with the reference's storage-type tree reduction
    (LaplaceSubtraction_cuda_kernel.cu:399-447, launcher :611-647)."""
    qn, name = _np(query)
    kn, _ = _np(key)
    B, H, N, M, D = _dims(qn, kn)
    if name == "float16":
        ct, tag = np.float16, "f16"
    elif name == "bfloat16":
        raise NotImplementedError("the reference has no bf16 reduce path")
    else:
        ct, tag = _compute_dtype(qn.dtype)
    q = np.ascontiguousarray(qn, dtype=ct)
    k = np.ascontiguousarray(kn, dtype=ct)
    s = np.empty((B, H, N, M), dtype=ct)
    fn = getattr(lib(), f"lfo_laplace_reduce_{tag}")
    jobs = [
        (lambda a=a, b=b: fn(_ptr(q, a * N * D), _ptr(k, a * D * M), _ptr(s, a * N * M), b - a, N, M, D))
        for a, b in _chunks(B * H)
    ]
    _run(jobs)
    return s


# --------------------------------------------------------------------------
# NewtonInverse
# --------------------------------------------------------------------------
INIT_REFERENCE = 0  # P = A + reg I, V0 = 1.8 / max_rowsum(P)^2 * P
INIT_SCALED_TRANSPOSE = 1  # X0 = A^T / (|A|_1 |A|_inf)


def reference_order(n: int, max_optin_smem: int = 232448) -> int:
    """Which association the reference kernel uses for V P V at size n.

    dispatch_forward (NewtonInverse_cuda_kernel.cu:693-728) runs the 3-buffer
    kernel, V (P V), whenever 3 * N_MAX * (N_MAX+1) * 4 bytes fit the device's
    opt-in shared memory and N_MAX < 128; N_MAX = 128 always takes the 2-buffer
    kernel, (V P) V.  On B200 (227 KB opt-in) every N_MAX <= 112 fits.
    """
    buckets = [16, 32, 48, 64, 80, 96, 112, 128]
    nmax = next(b for b in buckets if n <= b)
    if nmax == 128:
        return 1
    if nmax <= 80:
        return 0
    return 0 if 3 * nmax * (nmax + 1) * 4 <= max_optin_smem else 1


def newton_fwd(mat, iters: int, mode: int = INIT_REFERENCE, reg: float | None = None, order: int | None = None):
    """Newton–Schulz inverse of a batch of [N,N] matrices.

    mode INIT_REFERENCE follows NewtonInverse_cuda_kernel.cu:125-464 (reg
    defaults to the hard-coded 0.01 of :169); INIT_SCALED_TRANSPOSE is the
    X0 = A^T/(|A|_1|A|_inf), X <- X(2I - A X) variant (reg defaults to 0).
    """
    an, name = _np(mat)
    assert an.ndim >= 2 and an.shape[-1] == an.shape[-2]
    n = an.shape[-1]
    ct, tag = _compute_dtype(an.dtype)
    a = np.ascontiguousarray(an, dtype=ct)
    batch = int(np.prod(a.shape[:-2])) if a.ndim > 2 else 1
    x = np.empty_like(a)
    if reg is None:
        reg = 0.01 if mode == INIT_REFERENCE else 0.0
    if order is None:
        order = reference_order(n) if mode == INIT_REFERENCE else 1
    fn = getattr(lib(), f"lfo_newton_fwd_{tag}")
    jobs = [
        (lambda s=s, e=e: fn(_ptr(a, s * n * n), _ptr(x, s * n * n), e - s, n, int(iters), int(mode), ct(reg), int(order)))
        for s, e in _chunks(batch)
    ]
    _run(jobs)
    return _round_to(x, name)


def newton_bwd(grad, inverse):
    """dA = -(V^T G V^T) (NewtonInverse_cuda_kernel.cu:469-573)."""
    gn, _ = _np(grad)
    vn, name = _np(inverse)
    n = vn.shape[-1]
    ct, tag = _compute_dtype(vn.dtype)
    g = np.ascontiguousarray(gn, dtype=ct)
    v = np.ascontiguousarray(vn, dtype=ct)
    batch = int(np.prod(v.shape[:-2])) if v.ndim > 2 else 1
    da = np.empty_like(v)
    fn = getattr(lib(), f"lfo_newton_bwd_{tag}")
    jobs = [
        (lambda s=s, e=e: fn(_ptr(g, s * n * n), _ptr(v, s * n * n), _ptr(da, s * n * n), e - s, n))
        for s, e in _chunks(batch)
    ]
    _run(jobs)
    return _round_to(da, name)


def residual_fro(mat, inv, reg: float = 0.0):
    """||(A + reg I) X - I||_F per matrix, in float64."""
    a = np.asarray(_np(mat)[0], dtype=np.float64)
    x = np.asarray(_np(inv)[0], dtype=np.float64)
    n = a.shape[-1]
    eye = np.eye(n)
    r = (a + reg * eye) @ x - eye
    return np.sqrt((r * r).sum(axis=(-1, -2)))


# --------------------------------------------------------------------------
# Small pure-numpy restatements, used to cross-check the C code in tests.
# --------------------------------------------------------------------------
def np_laplace_fwd(q, k):
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    return np.abs(q[..., :, None, :] - np.swapaxes(k, -1, -2)[..., None, :, :]).sum(-1)


def np_laplace_bwd(g, q, k):
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    g = np.asarray(g, dtype=np.float64)
    sg = np.sign(q[..., :, None, :] - np.swapaxes(k, -1, -2)[..., None, :, :])  # [..,N,M,D]
    dq = (g[..., None] * sg).sum(-2)
    dk = -np.swapaxes((g[..., None] * sg).sum(-3), -1, -2)
    return dq, dk
