"""The CPU oracle (oracle/oracle.c) against independent numpy restatements,
the reference's documented edge behaviour, and the golden vectors produced by
the reference operators themselves (tests/golden/)."""
import glob
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _rng(seed=0):
    return np.random.default_rng(seed)


@pytest.mark.parametrize("shape", [(2, 3, 37, 24, 11), (1, 1, 5, 1, 1), (1, 2, 64, 33, 49)])
def test_forward_matches_numpy(shape):
    B, H, N, D, M = shape
    r = _rng(1)
    q = r.standard_normal((B, H, N, D)).astype(np.float32)
    k = r.standard_normal((B, H, D, M)).astype(np.float32)
    s = O.laplace_fwd(q, k)
    ref = O.np_laplace_fwd(q, k)
    assert s.shape == (B, H, N, M)
    np.testing.assert_allclose(s, ref, rtol=1e-5, atol=1e-5)


def test_forward_sequential_fp32_order():
    # The oracle must reproduce the reference's sequential-over-d fp32 sum
    # bit for bit: recompute it in numpy with explicit float32 steps.
    r = _rng(2)
    q = r.standard_normal((1, 1, 7, 19)).astype(np.float32)
    k = r.standard_normal((1, 1, 19, 5)).astype(np.float32)
    s = O.laplace_fwd(q, k)
    for i in range(7):
        for j in range(5):
            acc = np.float32(0)
            for c in range(19):
                acc = np.float32(acc + np.float32(abs(np.float32(q[0, 0, i, c] - k[0, 0, c, j]))))
            assert s[0, 0, i, j] == acc


def test_backward_matches_numpy():
    r = _rng(3)
    q = r.standard_normal((2, 2, 30, 9)).astype(np.float64)
    k = r.standard_normal((2, 2, 9, 13)).astype(np.float64)
    g = r.standard_normal((2, 2, 30, 13)).astype(np.float64)
    dq = O.laplace_bwd_query(g, q, k)
    dk = O.laplace_bwd_key(g, q, k)
    rq, rk = O.np_laplace_bwd(g, q, k)
    np.testing.assert_allclose(dq, rq, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(dk, rk, rtol=1e-12, atol=1e-12)


def test_backward_sign_of_zero_is_zero():
    # sign_func(0) = 0 (LaplaceSubtraction_cuda_kernel.cu:34-38): a query equal
    # to a landmark channel contributes nothing.
    q = np.array([[[[1.0, 2.0]]]], dtype=np.float32)       # [1,1,1,2]
    k = np.array([[[[1.0, 0.0], [2.0, 5.0]]]], dtype=np.float32)  # [1,1,2,2]
    g = np.array([[[[3.0, 7.0]]]], dtype=np.float32)
    dq = O.laplace_bwd_query(g, q, k)
    # channel 0: sign(1-1)=0, sign(1-0)=+1 -> 7 ; channel 1: sign(0)=0, sign(2-5)=-1 -> -7
    np.testing.assert_array_equal(dq.ravel(), [7.0, -7.0])
    dk = O.laplace_bwd_key(g, q, k)
    np.testing.assert_array_equal(dk.ravel(), [0.0, -7.0, 0.0, 7.0])


def test_reduce_power_of_two_equals_forward():
    r = _rng(4)
    q = r.standard_normal((1, 2, 9, 32)).astype(np.float32)
    k = r.standard_normal((1, 2, 32, 6)).astype(np.float32)
    np.testing.assert_allclose(O.laplace_reduce(q, k), O.laplace_fwd(q, k), rtol=1e-5)


def test_reduce_drops_partials_for_non_power_of_two():
    # blockDim = 48: the halving tree (24, 12, 6, 3, 1) never adds s[2] after
    # the stride-3 step (LaplaceSubtraction_cuda_kernel.cu:437-442).
    r = _rng(5)
    q = r.standard_normal((1, 1, 3, 48)).astype(np.float64)
    k = r.standard_normal((1, 1, 48, 2)).astype(np.float64)
    out = O.laplace_reduce(q, k)
    d = np.abs(q[0, 0, :, :, None] - k[0, 0][None])  # [3,48,2]
    part = d.copy()
    for st in (24, 12, 6, 3, 1):
        part[:, :st] = part[:, :st] + part[:, st:2 * st]
    np.testing.assert_allclose(out[0, 0], part[:, 0], rtol=1e-12)
    assert np.all(out[0, 0] < d.sum(1) - 1e-9)


def test_reduce_half_accumulates_in_half():
    r = _rng(6)
    q = (r.standard_normal((1, 1, 4, 64)) * 30).astype(np.float16)
    k = (r.standard_normal((1, 1, 64, 3)) * 30).astype(np.float16)
    out = O.laplace_reduce(q, k)
    assert out.dtype == np.float16
    exact = np.abs(q.astype(np.float64)[0, 0, :, :, None] - k.astype(np.float64)[0, 0][None]).sum(1)
    np.testing.assert_allclose(out[0, 0].astype(np.float64), exact, rtol=2e-3)


def _spd(batch, n, seed):
    r = _rng(seed)
    L = r.standard_normal((batch, n, 16))
    S = np.abs(L[:, :, None, :] - L[:, None, :, :]).sum(-1)
    return np.exp(-S / 4.0) + 1e-3 * np.eye(n)


@pytest.mark.parametrize("n", [16, 49, 64, 128])
def test_newton_reference_mode_converges(n):
    A = _spd(3, n, 7).astype(np.float64)
    X = O.newton_fwd(A, 40)
    res = O.residual_fro(A, X, 0.01)
    assert np.all(res < 1e-8), res


def test_newton_orders_agree_in_fp64():
    A = _spd(2, 32, 8)
    x0 = O.newton_fwd(A, 6, order=0)
    x1 = O.newton_fwd(A, 6, order=1)
    np.testing.assert_allclose(x0, x1, rtol=1e-10, atol=1e-12)


def test_newton_scaled_transpose_init():
    A = _spd(2, 24, 9)
    X = O.newton_fwd(A, 0, mode=O.INIT_SCALED_TRANSPOSE)
    n1 = np.abs(A).sum(-2).max(-1)
    ninf = np.abs(A).sum(-1).max(-1)
    np.testing.assert_allclose(X, np.swapaxes(A, -1, -2) / (n1 * ninf)[:, None, None], rtol=1e-12)
    X = O.newton_fwd(A, 30, mode=O.INIT_SCALED_TRANSPOSE)
    assert np.all(O.residual_fro(A, X) < 1e-8)


def test_newton_alpha_init_matches_reference_formula():
    A = _spd(1, 20, 10)
    X = O.newton_fwd(A, 0)
    P = A + 0.01 * np.eye(20)
    alpha = 1.8 / P.sum(-1).max() ** 2
    np.testing.assert_allclose(X, alpha * P, rtol=1e-12)


def test_newton_backward_matches_numpy():
    r = _rng(11)
    V = r.standard_normal((3, 17, 17))
    G = r.standard_normal((3, 17, 17))
    da = O.newton_bwd(G, V)
    Vt = np.swapaxes(V, -1, -2)
    np.testing.assert_allclose(da, -(Vt @ G @ Vt), rtol=1e-10, atol=1e-10)


def test_reference_order_matches_dispatch():
    # 3-buffer kernel (V(PV)) up to N_MAX = 112 on a 227 KB part, 2-buffer at 128.
    assert O.reference_order(49) == 0
    assert O.reference_order(112) == 0
    assert O.reference_order(113) == 1
    assert O.reference_order(128) == 1
    # A part with less than 152 KB of opt-in shared memory would run N_MAX = 112
    # on the 2-buffer kernel.
    assert O.reference_order(112, max_optin_smem=131072) == 1


# ---------------------------------------------------------------------------
# Golden vectors from the reference operators (see tests/golden/make_golden.py)
# ---------------------------------------------------------------------------
def _goldens(prefix):
    return sorted(glob.glob(os.path.join(GOLDEN, prefix + "*.npz")))


def test_golden_files_present():
    assert _goldens("laplace_"), "tests/golden/laplace_*.npz missing"
    assert _goldens("newton_"), "tests/golden/newton_*.npz missing"


@pytest.mark.parametrize("path", _goldens("laplace_"), ids=os.path.basename)
def test_oracle_matches_reference_golden_laplace(path):
    z = np.load(path)
    q, k, g = z["q"], z["k"], z["g"]
    dt = str(z["dtype"])
    if dt == "float16":
        q, k, g = q.astype(np.float16), k.astype(np.float16), g.astype(np.float16)
    s = O.laplace_fwd(q, k)
    # Forward: same fp32 operations in the same order -> identical bits
    # (inputs are N(0,1): no subnormal differences, so --use_fast_math's
    # flush-to-zero does not matter).
    np.testing.assert_array_equal(np.asarray(s, dtype=np.float64), z["s"].astype(np.float64))
    scale = np.abs(g.astype(np.float64)).sum(-1, keepdims=True)  # sum_j |g| per row
    tol = 1e-5 if dt != "float16" else 1e-2
    dq = np.asarray(O.laplace_bwd_query(g, q, k), dtype=np.float64)
    assert np.all(np.abs(dq - z["dq"]) <= tol * scale + 1e-6)
    colscale = np.abs(g.astype(np.float64)).sum(-2)[:, :, None, :]  # sum_i |g| per landmark
    dk = np.asarray(O.laplace_bwd_key(g, q, k), dtype=np.float64)
    assert np.all(np.abs(dk - z["dk"]) <= tol * colscale + 1e-6)
    r = O.laplace_reduce(q, k)
    if dt == "float16":
        np.testing.assert_array_equal(np.asarray(r).view(np.uint16), z["reduce"].astype(np.float16).view(np.uint16))
    else:
        np.testing.assert_array_equal(np.asarray(r, dtype=np.float64), z["reduce"].astype(np.float64))


@pytest.mark.parametrize("path", _goldens("newton_"), ids=os.path.basename)
def test_oracle_matches_reference_golden_newton(path):
    z = np.load(path)
    A, X, iters = z["A"], z["X"], int(z["iters"])
    Xo = O.newton_fwd(A.astype(np.float32), iters)
    rref = O.residual_fro(A, X, 0.01)
    ro = O.residual_fro(A, Xo, 0.01)
    assert np.all(np.abs(ro - rref) <= 1e-4), (ro, rref)
    np.testing.assert_allclose(Xo, X, rtol=2e-3, atol=2e-5 * np.abs(X).max())
    G, dA = z["G"], z["dA"]
    d = O.newton_bwd(G, X)
    np.testing.assert_allclose(d, dA, rtol=1e-4, atol=1e-5 * np.abs(dA).max())
