// NewtonInverse operator interface of the Laplace_subtraction_cuda extension,
// kept source-compatible with the reference header include/NewtonInverse.h
// (namespace laplace, same names, argument order and checks: CUDA, 4-D,
// square — reference NewtonInverse.h:22-47).  Implemented in
// laplacianformer_b200/csrc/torch_ops.cpp on top of laplacian_b200.h.
#pragma once
#include <torch/types.h>

namespace laplace {

void NewtonInverse_forward_cuda(const at::Tensor mat, at::Tensor output, int iter);
void NewtonInverse_backward_cuda(const at::Tensor grad_output, const at::Tensor inverse, at::Tensor grad_mat);
bool NewtonInverse_supports(int N);
// Extended forward (init mode, regulariser, arithmetic) and the per-matrix
// residual ||(A + reg I) X - I||_F.  No counterpart in the reference.
void NewtonInverse_forward_ex_cuda(const at::Tensor mat, at::Tensor output, int iter, int init_mode,
                                   double reg, int precision);
void NewtonInverse_residual_cuda(const at::Tensor mat, const at::Tensor inverse, at::Tensor residual, double reg);

inline void NewtonInverse_forward(const at::Tensor mat, at::Tensor output, int64_t iter) {
    TORCH_CHECK(mat.is_cuda(), "mat must be on GPU");
    TORCH_CHECK(mat.dim() == 4, "mat must be 4D (B,H,N,N)");
    TORCH_CHECK(mat.size(-1) == mat.size(-2), "last two dims of mat must be equal");
    NewtonInverse_forward_cuda(mat, output, static_cast<int>(iter));
}

inline void NewtonInverse_backward(const at::Tensor grad_output, const at::Tensor inverse, at::Tensor grad_mat) {
    TORCH_CHECK(grad_output.is_cuda() && inverse.is_cuda(), "tensors must be on GPU");
    TORCH_CHECK(grad_output.dim() == 4 && inverse.dim() == 4, "must be 4D");
    NewtonInverse_backward_cuda(grad_output, inverse, grad_mat);
}

inline bool NewtonInverse_is_supported(int64_t N) { return NewtonInverse_supports(static_cast<int>(N)); }

inline void NewtonInverse_forward_ex(const at::Tensor mat, at::Tensor output, int64_t iter, int64_t init_mode,
                                     double reg, int64_t precision) {
    TORCH_CHECK(mat.is_cuda(), "mat must be on GPU");
    TORCH_CHECK(mat.dim() == 4, "mat must be 4D (B,H,N,N)");
    TORCH_CHECK(mat.size(-1) == mat.size(-2), "last two dims of mat must be equal");
    NewtonInverse_forward_ex_cuda(mat, output, static_cast<int>(iter), static_cast<int>(init_mode), reg,
                                  static_cast<int>(precision));
}

inline void NewtonInverse_residual(const at::Tensor mat, const at::Tensor inverse, at::Tensor residual, double reg) {
    TORCH_CHECK(mat.is_cuda() && inverse.is_cuda() && residual.is_cuda(), "tensors must be on GPU");
    NewtonInverse_residual_cuda(mat, inverse, residual, reg);
}

}  // namespace laplace
