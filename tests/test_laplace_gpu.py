"""LaplaceSubtraction on the GPU, through the C ABI (liblfb200.so) and the
drop-in extension, against the CPU oracle and — where it was built — the
reference operators compiled for sm_100 (oracle/_ref)."""
import numpy as np
import pytest
import torch

from laplacianformer_b200 import capi
from oracle import oracle as O

pytestmark = pytest.mark.gpu

SHAPES = [
    # B, H, N, D, M
    (2, 2, 70, 32, 49),      # configuration-2 shape, scaled down
    (1, 3, 33, 17, 5),       # ragged channels / landmarks
    (1, 1, 1, 1, 1),         # minimum
    (1, 2, 600, 64, 64),     # d = 64, m = 64, several row tiles
    (1, 1, 37, 48, 9),       # non power-of-two channels
    (3, 1, 9, 100, 256),     # many landmarks, d > 64
    (1, 1, 1500, 8, 196),    # m = 196 (landmark-vs-key shape)
    (1, 2, 300, 64, 256),    # configuration-5 channels / landmarks (16-warp wide backward)
    (2, 1, 77, 40, 131),     # ragged channels and landmarks on the same path
]


def _inputs(shape, dtype, seed=0, device="cuda"):
    B, H, N, D, M = shape
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, N, D, generator=g).to(dtype)
    k = torch.randn(B, H, D, M, generator=g).to(dtype)
    gr = torch.randn(B, H, N, M, generator=g).to(dtype)
    return q, k, gr


def _np(t):
    return t.detach().cpu().to(torch.float64 if t.dtype == torch.float64 else torch.float32).numpy()


@pytest.mark.parametrize("shape", SHAPES, ids=str)
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.float16, torch.bfloat16], ids=str)
def test_forward_bit_exact_vs_oracle(cuda, shape, dtype):
    q, k, _ = _inputs(shape, dtype)
    s = capi.laplace_sub_fwd(q.to(cuda), k.to(cuda))
    torch.cuda.synchronize()
    ref = O.laplace_fwd(q, k)
    ref = ref.float().numpy() if isinstance(ref, torch.Tensor) else np.asarray(ref, dtype=np.float64)
    # Sequential fp32 (fp64) sum over channels, same operations as the
    # reference kernel, rounded once to the storage type: identical bits.
    np.testing.assert_array_equal(_np(s).astype(np.float64), np.asarray(ref, dtype=np.float64))


def _bwd_tol(dtype):
    return {torch.float32: 1e-5, torch.float64: 1e-12, torch.float16: 1e-2, torch.bfloat16: 1e-2}[dtype]


@pytest.mark.parametrize("shape", SHAPES, ids=str)
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.float16, torch.bfloat16], ids=str)
def test_backward_vs_oracle(cuda, shape, dtype):
    q, k, g = _inputs(shape, dtype, seed=1)
    dq, dk = capi.laplace_sub_bwd(g.to(cuda), q.to(cuda), k.to(cuda))
    dq_only = capi.laplace_sub_bwd_query(g.to(cuda), q.to(cuda), k.to(cuda))
    dk_only = capi.laplace_sub_bwd_key(g.to(cuda), q.to(cuda), k.to(cuda))
    torch.cuda.synchronize()
    rq = np.asarray(O.laplace_bwd_query(g.float() if dtype != torch.float64 else g, q.float() if dtype != torch.float64 else q, k.float() if dtype != torch.float64 else k), dtype=np.float64)
    rk = np.asarray(O.laplace_bwd_key(g.float() if dtype != torch.float64 else g, q.float() if dtype != torch.float64 else q, k.float() if dtype != torch.float64 else k), dtype=np.float64)
    ga = np.abs(_np(g).astype(np.float64))
    tol = _bwd_tol(dtype)
    # The reduction order differs from the reference, so the bound is
    # relative to the sum of |terms|: sum_j |g| per row for dQ, sum_i |g|
    # per landmark for dK.
    row = ga.sum(-1, keepdims=True)
    col = ga.sum(-2)[:, :, None, :]
    for got in (dq, dq_only):
        assert np.all(np.abs(_np(got) - rq) <= tol * row + 1e-30)
    for got in (dk, dk_only):
        assert np.all(np.abs(_np(got) - rk) <= tol * col + 1e-30)
    # dQ-only / dK-only kernels agree with the fused one
    np.testing.assert_allclose(_np(dq_only), _np(dq), rtol=0, atol=float(tol * row.max()))
    np.testing.assert_allclose(_np(dk_only), _np(dk), rtol=0, atol=float(tol * col.max()))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16], ids=str)
def test_backward_ties_give_zero_sign(cuda, dtype):
    # Queries equal to landmark values (the LaplaceSub(L, L^T) case) must use
    # sign(0) = 0 exactly.
    g0 = torch.Generator().manual_seed(5)
    L = torch.randn(2, 1, 24, 16, generator=g0).to(dtype)   # [B,H,M,D]
    q = L.clone()
    k = L.transpose(-1, -2).contiguous()
    g = torch.randn(2, 1, 24, 24, generator=g0).to(dtype)
    dq, dk = capi.laplace_sub_bwd(g.to(cuda), q.to(cuda), k.to(cuda))
    s = capi.laplace_sub_fwd(q.to(cuda), k.to(cuda))
    torch.cuda.synchronize()
    assert torch.all(torch.diagonal(s.float().cpu(), dim1=-2, dim2=-1) == 0)
    rq = O.laplace_bwd_query(g.float(), q.float(), k.float())
    rk = O.laplace_bwd_key(g.float(), q.float(), k.float())
    row = np.abs(_np(g)).sum(-1, keepdims=True)
    col = np.abs(_np(g)).sum(-2)[:, :, None, :]
    tol = _bwd_tol(dtype)
    assert np.all(np.abs(_np(dq) - np.asarray(rq, np.float64)) <= tol * row)
    assert np.all(np.abs(_np(dk) - np.asarray(rk, np.float64)) <= tol * col)


@pytest.mark.parametrize("shape", [(1, 2, 20, 32, 7), (1, 1, 11, 48, 5), (2, 1, 5, 300, 3), (1, 1, 4, 24, 3)], ids=str)
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.float16], ids=str)
def test_reduce_forward_bit_exact_vs_oracle(cuda, shape, dtype):
    q, k, _ = _inputs(shape, dtype, seed=2)
    r = capi.laplace_sub_reduce_fwd(q.to(cuda), k.to(cuda))
    torch.cuda.synchronize()
    ref = O.laplace_reduce(q.numpy() if dtype != torch.float16 else q.numpy(), k.numpy())
    got = r.cpu().numpy()
    if dtype == torch.float16:
        np.testing.assert_array_equal(got.view(np.uint16), np.asarray(ref).view(np.uint16))
    else:
        np.testing.assert_array_equal(got, ref)


def test_empty_and_degenerate(cuda):
    # empty batch / rows / landmarks: nothing to do, no error
    for B, H, N, D, M in [(0, 2, 5, 4, 3), (1, 1, 0, 4, 3), (1, 1, 5, 4, 0)]:
        q = torch.randn(B, H, N, D, device=cuda)
        k = torch.randn(B, H, D, M, device=cuda)
        g = torch.randn(B, H, N, M, device=cuda)
        s = capi.laplace_sub_fwd(q, k)
        dq, dk = capi.laplace_sub_bwd(g, q, k)
        assert s.shape == (B, H, N, M)
        if N == 0 and B * H > 0:
            assert torch.all(dk == 0)
    # d = 0: distances are 0
    q = torch.randn(1, 1, 5, 0, device=cuda)
    k = torch.randn(1, 1, 0, 3, device=cuda)
    s = capi.laplace_sub_fwd(q, k)
    assert torch.all(s == 0)


def test_large_offsets_64bit(cuda):
    # bh*n*m beyond 2^31 elements would overflow the reference's int offsets
    # (LaplaceSubtraction_cuda_kernel.cu:70-72); here the last (b,h) slice of
    # a 2^31+ element output is checked.  bh = 2, n = 2^20 + 1, m = 1024.
    bh, n, d, m = 2, (1 << 20) + 1, 4, 1024
    q = torch.randn(1, bh, n, d, device=cuda)
    k = torch.randn(1, bh, d, m, device=cuda)
    s = capi.laplace_sub_fwd(q, k)
    torch.cuda.synchronize()
    tail_q = q[:, 1:, -3:].cpu()
    ref = O.laplace_fwd(tail_q.numpy(), k[:, 1:].cpu().numpy())
    np.testing.assert_array_equal(s[:, 1:, -3:].cpu().numpy(), ref)
    del s


def test_canary_padding_untouched(cuda):
    # Outputs written through a view into a larger buffer must not spill.
    B, H, N, D, M = 1, 2, 45, 19, 13
    q, k, g = _inputs((B, H, N, D, M), torch.float32, seed=3)
    q, k, g = q.to(cuda), k.to(cuda), g.to(cuda)
    buf = torch.full((B * H * N * M + 64,), 12345.0, device=cuda)
    out = buf[32:32 + B * H * N * M].view(B, H, N, M)
    capi.laplace_sub_fwd(q, k, out)
    dqbuf = torch.full((B * H * N * D + 64,), 777.0, device=cuda)
    dkbuf = torch.full((B * H * D * M + 64,), 777.0, device=cuda)
    capi.laplace_sub_bwd(g, q, k, dqbuf[32:32 + B * H * N * D].view(B, H, N, D), dkbuf[32:32 + B * H * D * M].view(B, H, D, M))
    torch.cuda.synchronize()
    assert torch.all(buf[:32] == 12345.0) and torch.all(buf[-32:] == 12345.0)
    assert torch.all(dqbuf[:32] == 777.0) and torch.all(dqbuf[-32:] == 777.0)
    assert torch.all(dkbuf[:32] == 777.0) and torch.all(dkbuf[-32:] == 777.0)


def test_config2_full_size_properties(cuda):
    # Full configuration-2 size: bit-exact forward on sampled (b,h) slices,
    # and backward consistency between the fused and single-output kernels.
    from laplacianformer_b200 import workloads

    w = workloads.config2(device=cuda)
    q, kT, ds = w["q"], w["kT"], w["ds"]
    s = capi.laplace_sub_fwd(q, kT)
    dq, dk = capi.laplace_sub_bwd(ds, q, kT)
    torch.cuda.synchronize()
    for b, h in [(0, 0), (17, 1), (31, 1)]:
        ref = O.laplace_fwd(q[b:b + 1, h:h + 1].cpu().numpy(), kT[b:b + 1, h:h + 1].cpu().numpy())
        np.testing.assert_array_equal(s[b:b + 1, h:h + 1].cpu().numpy(), ref)
        rq = O.laplace_bwd_query(ds[b:b + 1, h:h + 1].cpu().numpy(), q[b:b + 1, h:h + 1].cpu().numpy(), kT[b:b + 1, h:h + 1].cpu().numpy())
        rk = O.laplace_bwd_key(ds[b:b + 1, h:h + 1].cpu().numpy(), q[b:b + 1, h:h + 1].cpu().numpy(), kT[b:b + 1, h:h + 1].cpu().numpy())
        ga = np.abs(ds[b:b + 1, h:h + 1].cpu().numpy().astype(np.float64))
        assert np.all(np.abs(dq[b:b + 1, h:h + 1].cpu().numpy() - rq) <= 1e-5 * ga.sum(-1, keepdims=True))
        assert np.all(np.abs(dk[b:b + 1, h:h + 1].cpu().numpy() - rk) <= 1e-5 * ga.sum(-2)[:, :, None, :])


def test_errors_are_reported(cuda):
    q = torch.randn(1, 1, 4, 3, device=cuda)
    k = torch.randn(1, 1, 3, 2, device=cuda)
    with pytest.raises(capi.LfError) as e:
        capi.lib()  # noqa: B018
        rc = capi.lib().lf_laplace_sub_fwd(q.data_ptr(), k.data_ptr(), q.data_ptr(), 1, 4, 2, 3, 9, None)
        capi._check(rc, "lf_laplace_sub_fwd")
    assert e.value.code == capi.LF_ERR_DTYPE
    rc = capi.lib().lf_laplace_sub_fwd(None, k.data_ptr(), q.data_ptr(), 1, 4, 2, 3, 0, None)
    assert rc == capi.LF_ERR_INVALID


# ---------------------------------------------------------------------------
# The drop-in extension (reference names and out-parameter contract)
# ---------------------------------------------------------------------------
def test_extension_ops_match_capi(cuda, ext):
    q, k, g = (t.to(cuda) for t in _inputs((2, 2, 70, 32, 49), torch.float32, seed=4))
    s = torch.empty(2, 2, 70, 49, device=cuda)
    ext.LaplaceSubtraction_forward(q, k, s)
    dq = torch.full_like(q, float("nan"))
    dk = torch.full_like(k, float("nan"))
    ext.LaplaceSubtraction_backward_query(g, q, k, dq)
    ext.LaplaceSubtraction_backward_key(g, q, k, dk)
    r = torch.empty_like(s)
    ext.LaplaceSubtraction_reduce_forward(q, k, r)
    torch.cuda.synchronize()
    assert torch.equal(s, capi.laplace_sub_fwd(q, k))
    dq2, dk2 = capi.laplace_sub_bwd(g, q, k)
    torch.testing.assert_close(dq, dq2, rtol=0, atol=1e-4)
    torch.testing.assert_close(dk, dk2, rtol=0, atol=1e-4)
    assert torch.equal(r, capi.laplace_sub_reduce_fwd(q, k))
    with pytest.raises(RuntimeError, match="query and key must match"):
        ext.LaplaceSubtraction_forward(q, k[:, :, :5].contiguous(), s)
    with pytest.raises(RuntimeError, match="contiguous"):
        ext.LaplaceSubtraction_forward(q.transpose(2, 3), k, s)
    with pytest.raises(RuntimeError, match=r"output has shape \[2, 2, 70, 48\]"):
        ext.LaplaceSubtraction_forward(q, k, s[..., :48].contiguous())


def test_autograd_function(cuda):
    from laplacianformer_b200.ops import laplace_subtraction

    g0 = torch.Generator().manual_seed(9)
    q = torch.randn(1, 2, 40, 8, generator=g0, dtype=torch.float64).to(cuda).requires_grad_()
    k = torch.randn(1, 2, 8, 6, generator=g0, dtype=torch.float64).to(cuda).requires_grad_()
    s = laplace_subtraction(q, k)
    ref = (q.detach()[..., :, None, :] - k.detach().transpose(-1, -2)[..., None, :, :]).abs().sum(-1)
    torch.testing.assert_close(s, ref)
    up = torch.randn_like(s)
    s.backward(up)
    qq = q.detach().clone().requires_grad_()
    kk = k.detach().clone().requires_grad_()
    (qq[..., :, None, :] - kk.transpose(-1, -2)[..., None, :, :]).abs().sum(-1).backward(up)
    torch.testing.assert_close(q.grad, qq.grad)
    torch.testing.assert_close(k.grad, kk.grad)


# ---------------------------------------------------------------------------
# Against the reference operators themselves (oracle/_ref), when built
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.float64], ids=str)
def test_against_reference_module(cuda, ref_module, dtype):
    if ref_module is None:
        pytest.skip("oracle/_ref not built (python oracle/build_ref.py)")
    from laplacianformer_b200 import workloads

    w = workloads.config2(device=cuda, dtype=dtype, batch=4)
    q, kT, ds = w["q"], w["kT"], w["ds"]
    s_ref = torch.empty(4, 2, 3136, 49, device=cuda, dtype=dtype)
    ref_module.LaplaceSubtraction_forward(q, kT, s_ref)
    s = capi.laplace_sub_fwd(q, kT)
    dq_ref = torch.empty_like(q)
    dk_ref = torch.empty_like(kT)
    ref_module.LaplaceSubtraction_backward_query(ds, q, kT, dq_ref)
    ref_module.LaplaceSubtraction_backward_key(ds, q, kT, dk_ref)
    dq, dk = capi.laplace_sub_bwd(ds, q, kT)
    torch.cuda.synchronize()
    assert torch.equal(s, s_ref)
    ga = ds.double().abs()
    row, col = ga.sum(-1, keepdim=True), ga.sum(-2).unsqueeze(-2)
    # fp16: the reference's own result is off by up to ~1.5e-2 * sum|dS|,
    # because its split-K paths add partials with atomicAdd in half precision
    # (LaplaceSubtraction_cuda_kernel.cu:260, :386), so the comparison with it
    # takes 2e-2; ours is held to the north-star 1e-2 against the oracle on
    # the same inputs below.
    tol = _bwd_tol(dtype) if dtype != torch.float16 else 2e-2
    assert torch.all((dq.double() - dq_ref.double()).abs() <= tol * row + 1e-30)
    assert torch.all((dk.double() - dk_ref.double()).abs() <= tol * col + 1e-30)
    if dtype == torch.float16:
        dsf, qf, kf = (t.float().cpu().numpy() for t in (ds, q, kT))
        oq = torch.from_numpy(np.asarray(O.laplace_bwd_query(dsf, qf, kf), dtype=np.float64)).to(cuda)
        ok = torch.from_numpy(np.asarray(O.laplace_bwd_key(dsf, qf, kf), dtype=np.float64)).to(cuda)
        assert torch.all((dq.double() - oq).abs() <= 1e-2 * row + 1e-30)
        assert torch.all((dk.double() - ok).abs() <= 1e-2 * col + 1e-30)


@pytest.mark.parametrize("shape,dtype,chunks", [
    ((3, 2, 130, 32, 49), torch.float32, 4),   # balanced backward per chunk, ragged last chunk
    ((7, 1, 70, 32, 49), torch.float16, 3),
    ((2, 1, 40, 20, 196), torch.float32, 5),   # workspace-free backward (m > 64)
    ((1, 2, 33, 17, 5), torch.bfloat16, 8),    # more chunks than slices
], ids=str)
def test_host_pipeline_matches_device_calls(cuda, shape, dtype, chunks):
    from laplacianformer_b200.streaming import HostPipeline

    B, H, N, D, M = shape
    q, k, g = _inputs(shape, dtype, seed=12)
    hq, hk, hg = q.pin_memory(), k.pin_memory(), g.pin_memory()
    hs = torch.empty(B, H, N, M, dtype=dtype).pin_memory()
    hdq = torch.empty_like(q).pin_memory()
    hdk = torch.empty_like(k).pin_memory()
    pipe = HostPipeline(q.shape, M, dtype=dtype, device=cuda, chunks=chunks)
    s = capi.laplace_sub_fwd(q.to(cuda), k.to(cuda))
    dq, dk = capi.laplace_sub_bwd(g.to(cuda), q.to(cuda), k.to(cuda))
    torch.cuda.synchronize()
    col = g.double().abs().sum(-2).unsqueeze(-2)
    for _ in range(2):  # buffer and stream reuse across calls
        hs.fill_(7.0), hdq.fill_(7.0), hdk.fill_(7.0)
        pipe(hq, hk, hg, hs, hdq, hdk)
        torch.cuda.synchronize()
        assert torch.equal(hs, s.cpu())
        assert torch.equal(hdq, dq.cpu())
        # dK^T partial sums are split per chunk: same value up to summation order
        assert torch.all((hdk.double() - dk.cpu().double()).abs() <= _bwd_tol(dtype) * col)


def test_host_pipeline_errors(cuda):
    L = capi.lib()
    need = L.lf_laplace_sub_host_buffer_size(4, 100, 49, 32, capi.LF_F32, 2)
    assert need > 0
    buf = torch.empty(need, dtype=torch.uint8, device=cuda)
    h = torch.empty(4 * 100 * 49).pin_memory()
    rc = L.lf_laplace_sub_fwd_bwd_host(h.data_ptr(), h.data_ptr(), h.data_ptr(), h.data_ptr(), h.data_ptr(),
                                       h.data_ptr(), 4, 100, 49, 32, capi.LF_F32, 2, buf.data_ptr(), need - 1, None)
    assert rc == capi.LF_ERR_INVALID and b"device buffer" in L.lf_last_error()


def _bwd_plain(g, q, k):
    """The workspace-free fused backward (per-(b,h) thread-block clusters)."""
    dq, dk = torch.empty_like(q), torch.empty_like(k)
    bh, n, m, d = q.shape[0] * q.shape[1], q.shape[2], k.shape[3], q.shape[3]
    assert capi.lib().lf_laplace_sub_bwd(g.data_ptr(), q.data_ptr(), k.data_ptr(), dq.data_ptr(), dk.data_ptr(),
                                         bh, n, m, d, capi.dtype_code(q), None) == capi.LF_OK
    return dq, dk


@pytest.mark.parametrize("shape", [
    (8, 40, 64, 32, 49),    # one row chunk per (b,h): a CTA spans many (b,h)
    (3, 7, 130, 16, 20),    # ragged last chunk, CTA ranges cross (b,h) mid-way
    (50, 3, 1, 32, 49),     # single query row
    (1, 1, 3000, 32, 64),   # one (b,h) split over many CTAs
    (4, 2, 3136, 32, 49),   # configuration-2 rows
    (3, 2, 700, 64, 256),   # configuration-5 channels / landmarks (16-warp wide kernel, balanced)
    (1, 3, 1000, 40, 131),  # ragged, same kernel
], ids=str)
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16], ids=str)
def test_balanced_backward_matches_oracle_and_cluster_kernel(cuda, shape, dtype):
    q, k, g = (t.to(cuda) for t in _inputs(shape, dtype, seed=3))
    need = capi.laplace_sub_bwd_workspace_size(q, k)
    assert need > 0
    ws = torch.full((need // 4,), float("nan"), device=cuda).view(torch.uint8)  # contents must not matter
    dq, dk = capi.laplace_sub_bwd(g, q, k, workspace=ws)
    dq2, dk2 = capi.laplace_sub_bwd(g, q, k, workspace=ws)
    pq, pk = _bwd_plain(g, q, k)
    torch.cuda.synchronize()
    assert torch.equal(dq, dq2) and torch.equal(dk, dk2)  # reproducible
    gf = g.float().cpu().numpy()
    ga = np.abs(gf.astype(np.float64))
    tol = _bwd_tol(dtype)
    row = ga.sum(-1, keepdims=True)
    col = ga.sum(-2)[:, :, None, :]
    rq = np.asarray(O.laplace_bwd_query(gf, q.float().cpu().numpy(), k.float().cpu().numpy()), dtype=np.float64)
    rk = np.asarray(O.laplace_bwd_key(gf, q.float().cpu().numpy(), k.float().cpu().numpy()), dtype=np.float64)
    assert np.all(np.abs(_np(dq) - rq) <= tol * row + 1e-30)
    assert np.all(np.abs(_np(dk) - rk) <= tol * col + 1e-30)
    # dQ is computed identically by both kernels; dK differs only in the
    # order of the partial sums.
    assert torch.equal(dq, pq)
    np.testing.assert_allclose(_np(dk), _np(pk), rtol=0, atol=float(tol * col.max()))


def test_balanced_backward_workspace_errors(cuda):
    q, k, g = (t.to(cuda) for t in _inputs((2, 2, 70, 32, 49), torch.float32))
    need = capi.laplace_sub_bwd_workspace_size(q, k)
    small = torch.empty(need - 16, dtype=torch.uint8, device=cuda)
    with pytest.raises(RuntimeError, match="workspace"):
        capi.laplace_sub_bwd(g, q, k, workspace=small)
    # shapes off the balanced path report no workspace and ignore it
    q2, k2, g2 = (t.to(cuda) for t in _inputs((1, 1, 9, 100, 256), torch.float32))
    assert capi.laplace_sub_bwd_workspace_size(q2, k2) == 0
    assert capi.laplace_sub_bwd_workspace_size(q.double(), k.double()) == 0


@pytest.mark.parametrize("shape", [(2, 2, 70, 32, 49), (1, 3, 33, 17, 5), (2, 1, 50, 64, 256), (1, 1, 9, 100, 20),
                                   (1, 1, 4, 0, 3)], ids=str)
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.float16, torch.bfloat16], ids=str)
def test_laplace_kernel_fused_exp(cuda, shape, dtype):
    """exp(scale*S) in the forward's store equals exp of the (bit-exact) S."""
    q, k, _ = _inputs(shape, dtype, seed=21)
    scale = -1.0 / 5.0
    got = capi.laplace_kernel_fwd(q.to(cuda), k.to(cuda), scale)
    torch.cuda.synchronize()
    if shape[3] == 0:
        assert torch.all(got.float() == 1.0)
        return
    wide = dtype in (torch.float16, torch.bfloat16)  # 16-bit inputs accumulate in fp32
    ref_s = np.asarray(O.laplace_fwd(q.float() if wide else q, k.float() if wide else k), dtype=np.float64)
    ref = np.exp(scale * ref_s)
    # expf of the fp32-rounded argument: a few ulp in fp32; one rounding to 16-bit types
    rtol = {torch.float32: 4e-6, torch.float64: 1e-14, torch.float16: 1e-3, torch.bfloat16: 8e-3}[dtype]
    atol = 6e-8 if dtype == torch.float16 else 0.0  # one fp16 subnormal step
    np.testing.assert_allclose(_np(got).astype(np.float64), ref, rtol=rtol, atol=atol)


def test_laplace_kernel_autograd_matches_composition(cuda):
    from laplacianformer_b200.ops import laplace_kernel, laplace_subtraction

    q, k, _ = _inputs((2, 2, 70, 32, 49), torch.float32, seed=22)
    q1, k1 = q.to(cuda).requires_grad_(), k.to(cuda).requires_grad_()
    q2, k2 = q.to(cuda).requires_grad_(), k.to(cuda).requires_grad_()
    g = torch.randn(2, 2, 70, 49, device=cuda)
    a = laplace_kernel(q1, k1, -0.2)
    b = torch.exp(-0.2 * laplace_subtraction(q2, k2))
    torch.testing.assert_close(a, b, rtol=4e-6, atol=0)
    (a * g).sum().backward()
    (b * g).sum().backward()
    torch.testing.assert_close(q1.grad, q2.grad, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(k1.grad, k2.grad, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("shape", [(2, 2, 70, 32, 49), (1, 3, 33, 17, 5), (2, 1, 196, 64, 49), (1, 2, 49, 64, 196),
                                   (1, 2, 300, 64, 256), (1, 1, 9, 100, 20)], ids=str)
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16], ids=str)
def test_laplace_kernel_backward_fused(cuda, shape, dtype):
    """dS = scale * Kmat * dKmat formed inside the backward kernel equals the
    LaplaceSub backward of that dS (computed in fp32 from the same stored
    values) within the backward tolerances, with and without workspace."""
    q, k, g = _inputs(shape, dtype, seed=21)
    qd, kd, gd = q.to(cuda), k.to(cuda), g.to(cuda)
    scale = -1.0 / 64.0  # keeps Kmat and the gradients in the normal range of fp16
    kmat = capi.laplace_kernel_fwd(qd, kd, scale)
    ds32 = (gd.float() * kmat.float()) * scale
    rq = np.asarray(O.laplace_bwd_query(ds32.cpu(), q.float(), k.float()), dtype=np.float64)
    rk = np.asarray(O.laplace_bwd_key(ds32.cpu(), q.float(), k.float()), dtype=np.float64)
    ga = np.abs(ds32.cpu().double().numpy())
    row, col = ga.sum(-1, keepdims=True), ga.sum(-2)[:, :, None, :]
    tol = _bwd_tol(dtype)
    need = capi.laplace_sub_bwd_workspace_size(qd, kd)
    ws = torch.full((max(need, 16) // 4,), float("nan"), device=cuda).view(torch.uint8) if need else None
    for workspace in (None, ws):
        dq, dk = capi.laplace_kernel_bwd(gd, kmat, qd, kd, scale, workspace=workspace)
        torch.cuda.synchronize()
        floor = {torch.float32: 1e-30, torch.float16: 2.0 ** -25, torch.bfloat16: 1e-30}[dtype]  # fp16 subnormal half-ulp
        assert np.all(np.abs(_np(dq) - rq) <= tol * row + floor)
        assert np.all(np.abs(_np(dk) - rk) <= tol * col + floor)


def test_laplace_kernel_autograd_uses_fused_backward(cuda):
    from laplacianformer_b200.ops import laplace_kernel

    q, k, g = _inputs((2, 2, 50, 32, 13), torch.float32, seed=22)
    qd = q.to(cuda).requires_grad_()
    kd = k.to(cuda).requires_grad_()
    out = laplace_kernel(qd, kd, -0.25)
    out.backward(g.to(cuda))
    q2 = q.double().requires_grad_()
    k2 = k.double().requires_grad_()
    ref = torch.exp(-0.25 * (q2[..., :, None, :] - k2.transpose(-1, -2)[..., None, :, :]).abs().sum(-1))
    ref.backward(g.double())
    torch.testing.assert_close(qd.grad.double().cpu(), q2.grad, rtol=0, atol=1e-5 * q2.grad.abs().max().item())
    torch.testing.assert_close(kd.grad.double().cpu(), k2.grad, rtol=0, atol=1e-5 * k2.grad.abs().max().item())


@pytest.mark.parametrize("shape", [(2, 2, 70, 32, 49), (1, 3, 33, 17, 5), (1, 1, 1, 1, 1), (1, 2, 600, 64, 64),
                                   (1, 1, 300, 16, 196), (1, 2, 300, 64, 256), (2, 1, 77, 40, 131),
                                   (32, 2, 3136, 32, 49)], ids=str)
def test_packed_fp16_forward_within_half_tolerance(cuda, shape):
    """The opt-in packed-half2 forward against the oracle's fp32 channel sums
    of the same fp16 inputs: relative error within the 1e-2 of the
    half-precision path (measured ~1e-3), exact zeros where q = k."""
    q, k, _ = _inputs(shape, torch.float16, seed=3)
    s = capi.laplace_sub_fwd_packed(q.cuda(), k.cuda())
    torch.cuda.synchronize()
    ref = np.asarray(O.laplace_fwd(q.float(), k.float()), dtype=np.float64)  # fp32 sums of the fp16 values
    got = s.double().cpu().numpy()
    assert np.all(np.abs(got - ref) <= 1e-2 * np.abs(ref) + 1e-3), np.max(np.abs(got - ref) / (np.abs(ref) + 1e-3))
    # the same query rows as landmarks give zero distances on the diagonal
    B, H, N, D, M = shape
    if N >= M:
        kq = q[:, :, :M, :].transpose(-1, -2).contiguous()
        s2 = capi.laplace_sub_fwd_packed(q.cuda(), kq.cuda())
        torch.cuda.synchronize()
        diag = torch.diagonal(s2[:, :, :M, :], dim1=-2, dim2=-1)
        assert torch.all(diag == 0)


def test_packed_fp16_forward_rejects_other_dtypes(cuda):
    q, k, _ = _inputs((1, 1, 8, 8, 4), torch.float32)
    with pytest.raises(RuntimeError):
        capi.laplace_sub_fwd_packed(q.cuda(), k.cuda())
    q, k, _ = _inputs((1, 1, 8, 65, 4), torch.float16)
    with pytest.raises(RuntimeError):
        capi.laplace_sub_fwd_packed(q.cuda(), k.cuda())
