"""NewtonInverse on the GPU (tcgen05 split-fp16 path and CUDA-core path)
against the CPU oracle and, where built, the reference operators."""
import numpy as np
import pytest
import torch

from laplacianformer_b200 import capi
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def spd(batch, n, seed, d=16, sigma=4.0, ridge=1e-3):
    g = torch.Generator().manual_seed(seed)
    L = torch.randn(batch, n, d, generator=g, dtype=torch.float64)
    A = torch.exp(-torch.cdist(L, L, p=1) / sigma) + ridge * torch.eye(n, dtype=torch.float64)
    return A.float().view(1, batch, n, n)


def _res(A, X, reg):
    return O.residual_fro(np.asarray(A, np.float64), np.asarray(X, np.float64), reg)


@pytest.mark.parametrize("n", [1, 7, 16, 49, 64, 100, 127, 128])
@pytest.mark.parametrize("mode", [capi.INIT_REFERENCE, capi.INIT_SCALED_TRANSPOSE])
def test_forward_split3_vs_oracle(cuda, n, mode):
    A = spd(6, n, seed=n)
    iters = 12
    reg = 0.01 if mode == capi.INIT_REFERENCE else 0.0
    X = capi.newton_inverse_fwd(A.to(cuda), iters, init_mode=mode)
    torch.cuda.synchronize()
    assert capi.device_status() == 0
    Xr = O.newton_fwd(A.numpy(), iters, mode=mode)
    r_gpu = _res(A.numpy(), X.cpu().numpy(), reg)
    r_ref = _res(A.numpy(), Xr, reg)
    # residual within 1e-4 of the reference's
    assert np.all(np.abs(r_gpu - r_ref) <= 1e-4), (r_gpu, r_ref)
    scale = np.abs(Xr).max()
    np.testing.assert_allclose(X.cpu().numpy(), Xr, rtol=0, atol=1e-4 * scale)


def test_reference_entry_point_defaults(cuda):
    A = spd(4, 128, seed=3).to(cuda)
    X1 = capi.newton_inverse_fwd_reference(A, 12)
    X2 = capi.newton_inverse_fwd(A, 12, init_mode=capi.INIT_REFERENCE, reg=0.01, precision=capi.PREC_SPLIT3)
    torch.cuda.synchronize()
    assert torch.equal(X1, X2)


def test_config3_batch_residual(cuda):
    # Configuration-3 matrices (128x128, sigma = 8, 1e-3 ridge), a 256-matrix
    # slice, scaled-transpose init, 12 iterations: every matrix against the oracle.
    from laplacianformer_b200 import workloads

    A = workloads.config3(device=cuda, batch=256)["A"]
    An = A.cpu().numpy()
    Xr = O.newton_fwd(An, 12, mode=O.INIT_SCALED_TRANSPOSE)
    r_ref = _res(An, Xr, 0.0).ravel()
    for prec in (capi.PREC_SPLIT3, capi.PREC_MIXED):
        X = capi.newton_inverse_fwd(A, 12, init_mode=capi.INIT_SCALED_TRANSPOSE, precision=prec)
        res = capi.newton_inverse_residual(A, X, 0.0)
        torch.cuda.synchronize()
        r_gpu = _res(An, X.cpu().numpy(), 0.0).ravel()
        assert np.all(np.abs(r_gpu - r_ref) <= 1e-4), (prec, np.abs(r_gpu - r_ref).max())
        # the device residual kernel agrees with the host computation
        np.testing.assert_allclose(res.reshape(-1).cpu().numpy(), r_gpu, rtol=1e-2, atol=1e-5)


def test_config3_full_batch_vs_oracle(cuda):
    # The whole configuration-3 batch (4096 matrices), drop-in entry point
    # (reference init, A + 0.01 I), every residual within 1e-4 of the oracle's.
    from laplacianformer_b200 import workloads

    A = workloads.config3(device=cuda, batch=4096)["A"]
    X = capi.newton_inverse_fwd_reference(A, 12)
    torch.cuda.synchronize()
    An = A.cpu().numpy()
    Xr = O.newton_fwd(An, 12)
    r_ref = _res(An, Xr, 0.01).ravel()
    r_gpu = _res(An, X.cpu().numpy(), 0.01).ravel()
    assert r_gpu.size == 4096
    assert np.all(np.abs(r_gpu - r_ref) <= 1e-4), np.abs(r_gpu - r_ref).max()


@pytest.mark.parametrize("n", [5, 64, 128])
def test_fp32_simt_mode(cuda, n):
    A = spd(3, n, seed=40 + n)
    X = capi.newton_inverse_fwd(A.to(cuda), 10, precision=capi.PREC_FP32_SIMT)
    torch.cuda.synchronize()
    Xr = O.newton_fwd(A.numpy(), 10, order=1)
    np.testing.assert_allclose(X.cpu().numpy(), Xr, rtol=0, atol=2e-5 * np.abs(Xr).max())


@pytest.mark.parametrize("n", [3, 64, 112, 128])
def test_fp64(cuda, n):
    A = spd(2, n, seed=60 + n).double()
    X = capi.newton_inverse_fwd(A.to(cuda), 9)
    torch.cuda.synchronize()
    Xr = O.newton_fwd(A.numpy(), 9, order=1)
    np.testing.assert_allclose(X.cpu().numpy(), Xr, rtol=1e-10, atol=1e-12 * np.abs(Xr).max())


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=str)
def test_half_inputs(cuda, dtype):
    A = spd(4, 49, seed=7)
    Ah = A.to(dtype)
    X = capi.newton_inverse_fwd(Ah.to(cuda), 8)
    torch.cuda.synchronize()
    Xr = O.newton_fwd(Ah.float().numpy(), 8)
    Xr_t = torch.from_numpy(np.ascontiguousarray(Xr)).to(dtype).float().numpy()
    np.testing.assert_allclose(X.float().cpu().numpy(), Xr_t, rtol=2e-2, atol=2e-2 * np.abs(Xr).max())


def test_zero_iterations_returns_init(cuda):
    A = spd(2, 30, seed=8)
    X = capi.newton_inverse_fwd(A.to(cuda), 0)
    torch.cuda.synchronize()
    np.testing.assert_allclose(X.cpu().numpy(), O.newton_fwd(A.numpy(), 0), rtol=1e-6, atol=1e-9)


@pytest.mark.parametrize("n", [1, 33, 128])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.float16], ids=str)
def test_backward_vs_oracle(cuda, n, dtype):
    g0 = torch.Generator().manual_seed(n)
    V = torch.randn(2, 3, n, n, generator=g0, dtype=torch.float64).to(dtype)
    G = torch.randn(2, 3, n, n, generator=g0, dtype=torch.float64).to(dtype)
    dA = capi.newton_inverse_bwd(G.to(cuda), V.to(cuda))
    torch.cuda.synchronize()
    wide = torch.float64 if dtype == torch.float64 else torch.float32
    ref = O.newton_bwd(G.to(wide).numpy(), V.to(wide).numpy())
    tol = {torch.float32: 1e-5, torch.float64: 1e-12, torch.float16: 1e-2}[dtype]
    scale = np.abs(ref).max() + 1e-30
    np.testing.assert_allclose(dA.to(wide).cpu().numpy(), np.asarray(torch.tensor(ref).to(dtype).to(wide)), rtol=0, atol=tol * scale * 4)


def test_unsupported_sizes(cuda):
    assert capi.newton_inverse_supported(256)
    assert not capi.newton_inverse_supported(257)
    A = torch.randn(1, 1, 257, 257, device=cuda)
    with pytest.raises(capi.LfError) as e:
        capi.newton_inverse_fwd(A, 3)
    assert e.value.code == capi.LF_ERR_UNSUPPORTED
    # beyond 128 only fp32 (the iterate is kept in the output buffer)
    with pytest.raises(capi.LfError) as e:
        capi.newton_inverse_fwd(torch.randn(1, 1, 200, 200, device=cuda).half(), 3)
    assert e.value.code == capi.LF_ERR_UNSUPPORTED


@pytest.mark.parametrize("n", [129, 200, 256])
@pytest.mark.parametrize("mode", [capi.INIT_REFERENCE, capi.INIT_SCALED_TRANSPOSE])
def test_forward_large_n(cuda, n, mode):
    # 128 < n <= 256 (configuration 5's landmark kernel): two-CTA cluster path.
    A = spd(2, n, seed=n)
    X = capi.newton_inverse_fwd(A.to(cuda), 10, init_mode=mode)
    torch.cuda.synchronize()
    Xr = O.newton_fwd(A.numpy(), 10, mode=mode, order=1)
    reg = 0.01 if mode == capi.INIT_REFERENCE else 0.0
    r_gpu = _res(A.numpy(), X.cpu().numpy(), reg)
    r_ref = _res(A.numpy(), Xr, reg)
    assert np.all(np.abs(r_gpu - r_ref) <= 1e-4), (r_gpu, r_ref)
    np.testing.assert_allclose(X.cpu().numpy(), Xr, rtol=0, atol=1e-4 * np.abs(Xr).max())


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64], ids=str)
def test_backward_large_n(cuda, dtype):
    g0 = torch.Generator().manual_seed(3)
    V = torch.randn(1, 2, 256, 256, generator=g0, dtype=torch.float64).to(dtype)
    G = torch.randn(1, 2, 256, 256, generator=g0, dtype=torch.float64).to(dtype)
    dA = capi.newton_inverse_bwd(G.to(cuda), V.to(cuda))
    torch.cuda.synchronize()
    ref = O.newton_bwd(G.numpy(), V.numpy())
    tol = 1e-5 if dtype == torch.float32 else 1e-12
    np.testing.assert_allclose(dA.cpu().numpy(), ref, rtol=0, atol=tol * 4 * np.abs(ref).max())


def test_extension_and_autograd(cuda, ext):
    from laplacianformer_b200.ops import newton_inverse

    A = spd(1, 64, seed=11).to(cuda)
    out = torch.empty_like(A)
    ext.NewtonInverse_forward(A, out, 10)
    assert torch.equal(out, capi.newton_inverse_fwd_reference(A, 10))
    assert ext.NewtonInverse_is_supported(256) and not ext.NewtonInverse_is_supported(257)
    with pytest.raises(RuntimeError, match="not supported"):
        big = torch.randn(1, 1, 260, 260, device=cuda)
        ext.NewtonInverse_forward(big, torch.empty_like(big), 3)
    Ad = A.double().requires_grad_()
    X = newton_inverse(Ad, 30)
    G = torch.randn_like(X)
    X.backward(G)
    Xd = X.detach()
    expect = -(Xd.transpose(-1, -2) @ G @ Xd.transpose(-1, -2))
    torch.testing.assert_close(Ad.grad, expect)


def test_against_reference_module(cuda, ref_module):
    if ref_module is None:
        pytest.skip("oracle/_ref not built (python oracle/build_ref.py)")
    for n, iters in ((64, 10), (128, 12), (49, 8)):
        A = spd(8, n, seed=100 + n).to(cuda)
        Xr = torch.empty_like(A)
        ref_module.NewtonInverse_forward(A, Xr, iters)
        X = capi.newton_inverse_fwd_reference(A, iters)
        G = torch.randn_like(A)
        dr = torch.empty_like(A)
        ref_module.NewtonInverse_backward(G, Xr, dr)
        d = capi.newton_inverse_bwd(G, Xr)
        torch.cuda.synchronize()
        r_ref = _res(A.cpu().numpy(), Xr.cpu().numpy(), 0.01)
        r_gpu = _res(A.cpu().numpy(), X.cpu().numpy(), 0.01)
        assert np.all(np.abs(r_gpu - r_ref) <= 1e-4), (n, r_gpu, r_ref)
        torch.testing.assert_close(X, Xr, rtol=0, atol=1e-4 * Xr.abs().max().item())
        torch.testing.assert_close(d, dr, rtol=0, atol=1e-5 * dr.abs().max().item())


def test_bounded_wait_reports_timeout(cuda):
    # A device wait that nothing completes gives up after its limit and
    # reports LF_ERR_TIMEOUT through the status word; the context stays usable.
    assert capi.device_status(clear=True) in (0, capi.LF_ERR_TIMEOUT)
    assert capi.device_status() == 0
    s = torch.cuda.current_stream(cuda).cuda_stream
    assert capi.lib().lf_selftest_bounded_wait(50, s) == capi.LF_OK
    assert capi.device_status(clear=True) == capi.LF_ERR_TIMEOUT
    assert capi.device_status() == 0
    # still usable afterwards
    A = spd(2, 64, seed=1).to(cuda)
    X = capi.newton_inverse_fwd(A, 10)
    torch.cuda.synchronize()
    assert torch.isfinite(X).all()


@pytest.mark.parametrize("n,d", [(49, 64), (128, 64), (17, 5), (100, 128)], ids=str)
@pytest.mark.parametrize("init_mode", [capi.INIT_REFERENCE, capi.INIT_SCALED_TRANSPOSE], ids=str)
def test_landmark_inverse_fused_equals_two_step(cuda, n, d, init_mode):
    """A = exp(scale*S_LL) built inside the inverse kernel gives the same bits
    as lf_laplace_kernel_fwd followed by the inverse of that stored A."""
    g = torch.Generator().manual_seed(n * 1000 + d)
    L = torch.randn(3, 2, n, d, generator=g).to(cuda)
    scale = -1.0 / (d ** 0.5)
    A = capi.laplace_kernel_fwd(L, L.transpose(-1, -2).contiguous(), scale)
    for prec in (capi.PREC_SPLIT3, capi.PREC_MIXED):
        x2 = capi.newton_inverse_fwd(A, 10, init_mode=init_mode, precision=prec)
        x1 = capi.laplace_newton_inverse_fwd(L, scale, 10, init_mode=init_mode, precision=prec)
        torch.cuda.synchronize()
        assert torch.equal(x1, x2)


def test_landmark_inverse_fused_rejects_unsupported(cuda):
    L = torch.randn(1, 129, 8, device=cuda)
    with pytest.raises(RuntimeError, match="n <= 128"):
        capi.laplace_newton_inverse_fwd(L, -0.1, 5)
    L = torch.randn(1, 16, 8, device=cuda)
    with pytest.raises(RuntimeError, match="precision"):
        capi.laplace_newton_inverse_fwd(L, -0.1, 5, precision=capi.PREC_FP32_SIMT)


@pytest.mark.parametrize("n", [5, 49, 64, 100])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=str)
def test_backward_tensor_core_packed_tiles(cuda, n, dtype):
    # n <= 64 packs floor(128/n) matrices per tile (per-matrix scales); a
    # ragged last tile (batch not a multiple of the packing) is included.
    g0 = torch.Generator().manual_seed(200 + n)
    batch = 7
    V = (torch.randn(1, batch, n, n, generator=g0, dtype=torch.float64) * torch.logspace(-3, 3, batch, dtype=torch.float64).view(1, batch, 1, 1)).to(dtype)
    G = torch.randn(1, batch, n, n, generator=g0, dtype=torch.float64).to(dtype)
    dA = capi.newton_inverse_bwd(G.to(cuda), V.to(cuda))
    torch.cuda.synchronize()
    ref = O.newton_bwd(G.float().numpy(), V.float().numpy())
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    for b in range(batch):  # per matrix: magnitudes differ by 10^6 across the batch
        r = ref[0, b]
        np.testing.assert_allclose(dA[0, b].float().cpu().numpy(), r, rtol=0, atol=tol * 4 * np.abs(r).max())


@pytest.mark.parametrize("n", [129, 256])
def test_forward_large_n_mixed_zero_iters_and_simt(cuda, n):
    A = spd(3, n, seed=300 + n)
    Ad = A.to(cuda)
    X0 = capi.newton_inverse_fwd(Ad, 0)
    torch.cuda.synchronize()
    np.testing.assert_allclose(X0.cpu().numpy(), O.newton_fwd(A.numpy(), 0, order=1), rtol=1e-6, atol=1e-9)
    Xr = O.newton_fwd(A.numpy(), 10, order=1)
    r_ref = _res(A.numpy(), Xr, 0.01)
    for prec in (capi.PREC_MIXED, capi.PREC_FP32_SIMT):
        X = capi.newton_inverse_fwd(Ad, 10, precision=prec)
        torch.cuda.synchronize()
        assert capi.device_status() == 0
        r_gpu = _res(A.numpy(), X.cpu().numpy(), 0.01)
        assert np.all(np.abs(r_gpu - r_ref) <= 1e-4), (prec, r_gpu, r_ref)
