"""CPU-side checks of the drop-in boundary: the C-ABI library loads and
exports every entry point include/laplacian_b200.h declares, the PyTorch
extension keeps the reference's module and operator names, and CPU tensors
fail the way the reference's do (no CPU fallback)."""
import ctypes
import os
import re

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "laplacian_b200.h")).read()
    return sorted(set(re.findall(r"^LF_API\s+[\w\s\*]+?\b(lf_\w+)\s*\(", src, flags=re.M)))


def test_header_declares_entry_points():
    names = _declared()
    for must in ("lf_laplace_sub_fwd", "lf_laplace_sub_bwd_query", "lf_laplace_sub_bwd_key", "lf_laplace_sub_bwd",
                 "lf_laplace_sub_reduce_fwd", "lf_newton_inverse_fwd", "lf_newton_inverse_fwd_ex",
                 "lf_newton_inverse_bwd", "lf_newton_inverse_supported", "lf_last_error"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from laplacianformer_b200 import capi

    lib = ctypes.CDLL(capi.LIB_PATH)
    for name in _declared():
        assert hasattr(lib, name), name
    # the ctypes table covers the header exactly
    assert set(capi.SIGNATURES) == set(_declared())


def test_host_only_entry_points():
    from laplacianformer_b200 import capi

    L = capi.lib()
    assert L.lf_cudart_version() >= 12000
    assert L.lf_version() >= 100
    assert capi.newton_inverse_supported(1) and capi.newton_inverse_supported(128)
    assert capi.newton_inverse_supported(256)
    assert not capi.newton_inverse_supported(0) and not capi.newton_inverse_supported(257)
    # argument validation happens before any device work
    assert L.lf_laplace_sub_fwd(None, None, None, 1, 2, 3, 4, 7, None) == capi.LF_ERR_DTYPE
    assert b"dtype" in L.lf_last_error()
    assert L.lf_laplace_sub_fwd(None, None, None, 1, 2, 3, 4, 0, None) == capi.LF_ERR_INVALID
    assert L.lf_laplace_sub_fwd(None, None, None, -1, 2, 3, 4, 0, None) == capi.LF_ERR_INVALID
    assert L.lf_newton_inverse_fwd(None, None, 1, 257, 3, 0, None) == capi.LF_ERR_UNSUPPORTED
    assert L.lf_newton_inverse_fwd_ex(None, None, 1, 4, 3, 0, 7, 0.0, 0, None) == capi.LF_ERR_INVALID
    # the packed forward is fp16 only and d <= 64
    assert L.lf_laplace_sub_fwd_packed(None, None, None, 1, 2, 3, 4, capi.LF_F32, None) == capi.LF_ERR_DTYPE
    assert L.lf_laplace_sub_fwd_packed(None, None, None, 1, 2, 3, 4, capi.LF_F16, None) == capi.LF_ERR_INVALID
    assert L.lf_laplace_sub_fwd_packed(None, None, None, 0, 2, 3, 4, capi.LF_F16, None) == capi.LF_OK
    # empty problems are no-ops
    assert L.lf_laplace_sub_fwd(None, None, None, 0, 2, 3, 4, 0, None) == capi.LF_OK
    assert L.lf_newton_inverse_fwd(None, None, 0, 64, 3, 0, None) == capi.LF_OK


def test_extension_keeps_reference_names():
    import Laplace_subtraction_cuda as L

    for name in ("LaplaceSubtraction_forward", "LaplaceSubtraction_backward_query", "LaplaceSubtraction_backward_key",
                 "LaplaceSubtraction_reduce_forward", "NewtonInverse_forward", "NewtonInverse_backward",
                 "NewtonInverse_is_supported", "get_compiler_version", "get_cuda_version", "has_cuda"):
        assert hasattr(L, name), name
    assert L.has_cuda()
    assert L.get_cuda_version().startswith("CUDA 12.")
    assert L.get_compiler_version()
    assert L.NewtonInverse_is_supported(256) and not L.NewtonInverse_is_supported(257)


def test_cpu_tensors_raise_like_the_reference():
    import Laplace_subtraction_cuda as L

    q = torch.zeros(1, 1, 4, 3)
    k = torch.zeros(1, 1, 3, 2)
    s = torch.zeros(1, 1, 4, 2)
    with pytest.raises(RuntimeError, match="Not implemented on the CPU"):
        L.LaplaceSubtraction_forward(q, k, s)
    with pytest.raises(RuntimeError, match="Not implemented on the CPU"):
        L.LaplaceSubtraction_backward_query(s, q, k, q.clone())
    with pytest.raises(RuntimeError, match="Not implemented on the CPU"):
        L.LaplaceSubtraction_backward_key(s, q, k, k.clone())
    with pytest.raises(RuntimeError, match="Not implemented on the CPU"):
        L.LaplaceSubtraction_reduce_forward(q, k, s)
    m = torch.zeros(1, 1, 4, 4)
    with pytest.raises(RuntimeError, match="mat must be on GPU"):
        L.NewtonInverse_forward(m, m.clone(), 3)
    with pytest.raises(RuntimeError, match="tensors must be on GPU"):
        L.NewtonInverse_backward(m, m, m.clone())


def test_ops_have_no_cpu_fallback():
    from laplacianformer_b200.ops import laplace_subtraction, newton_inverse

    with pytest.raises(RuntimeError):
        laplace_subtraction(torch.zeros(1, 1, 4, 3), torch.zeros(1, 1, 3, 2))
    with pytest.raises(RuntimeError):
        newton_inverse(torch.eye(4).view(1, 1, 4, 4), 3)
    from laplacianformer_b200 import capi

    with pytest.raises(RuntimeError, match="CUDA"):
        capi.laplace_sub_fwd(torch.zeros(1, 1, 4, 3), torch.zeros(1, 1, 3, 2))


def test_workload_shapes():
    from laplacianformer_b200 import workloads

    w = workloads.config1()
    assert w["q"].shape == (1, 1, 1024, 32) and w["kT"].shape == (1, 1, 32, 64) and w["A"].shape == (1, 1, 64, 64)
    w = workloads.config2(batch=2)
    assert w["q"].shape == (2, 2, 3136, 32) and w["kT"].shape == (2, 2, 32, 49) and w["ds"].shape == (2, 2, 3136, 49)
    w = workloads.config3(batch=128, n=16)
    assert w["A"].shape == (2, 64, 16, 16)
    assert torch.allclose(w["A"], w["A"].transpose(-1, -2))
    w = workloads.config4(batch=2)
    assert w["landmarks"].shape == (2, 8, 49, 64) and w["q"].dtype == torch.bfloat16
    w = workloads.config5(1024, batch=1, heads=2)
    assert w["kT"].shape == (1, 2, 64, 256)
    # seeded: identical on a second draw
    assert torch.equal(workloads.config2(batch=1)["q"], workloads.config2(batch=1)["q"])
