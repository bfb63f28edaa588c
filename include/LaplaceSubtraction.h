// LaplaceSubtraction operator interface of the Laplace_subtraction_cuda
// extension, kept source-compatible with the reference header
// include/LaplaceSubtraction.h (namespace laplace, same function names and
// argument order).  The *_cuda functions are implemented in
// laplacianformer_b200/csrc/torch_ops.cpp on top of the C ABI in
// laplacian_b200.h; the inline front ends dispatch on the device exactly like
// the reference: CUDA tensors go to the B200 kernels, anything else raises
// "Not implemented on the CPU" (reference LaplaceSubtraction.h:37-51).
#pragma once
#include <torch/types.h>

namespace laplace {

// Reference LaplaceSubtraction.h:8-33 (same four entry points).
void LaplaceSubtraction_forward_cuda(const at::Tensor query, const at::Tensor key, at::Tensor output);
void LaplaceSubtraction_backward_query_cuda(const at::Tensor gradOutput, const at::Tensor query,
                                            const at::Tensor key, at::Tensor gradQuery);
void LaplaceSubtraction_backward_key_cuda(const at::Tensor gradOutput, const at::Tensor query,
                                          const at::Tensor key, at::Tensor gradKey);
void LaplaceSubtraction_reduce_forward_cuda(const at::Tensor query, const at::Tensor key, at::Tensor output);
// Both gradients from one pass over gradOutput (either may be undefined).
// No counterpart in the reference.
void LaplaceSubtraction_backward_cuda(const at::Tensor gradOutput, const at::Tensor query,
                                      const at::Tensor key, at::Tensor gradQuery, at::Tensor gradKey);

// output = exp(scale * LaplaceSub(query, key)) in one pass (S not stored).
// No counterpart in the reference.
void LaplaceKernel_forward_cuda(const at::Tensor query, const at::Tensor key, at::Tensor output, double scale);

inline void LaplaceKernel_forward(const at::Tensor query, const at::Tensor key, at::Tensor output, double scale) {
    if (query.is_cuda() && key.is_cuda()) return LaplaceKernel_forward_cuda(query, key, output, scale);
    AT_ERROR("Not implemented on the CPU");
}

// Gradients of output = exp(scale * LaplaceSub(query, key)) from gradOutput:
// dS = scale * output * gradOutput is formed inside the backward kernel
// (never stored).  Either gradient may be undefined.  No counterpart in the
// reference.
void LaplaceKernel_backward_cuda(const at::Tensor gradOutput, const at::Tensor output, double scale,
                                 const at::Tensor query, const at::Tensor key, at::Tensor gradQuery,
                                 at::Tensor gradKey);

inline void LaplaceKernel_backward(const at::Tensor gradOutput, const at::Tensor output, double scale,
                                   const at::Tensor query, const at::Tensor key, at::Tensor gradQuery,
                                   at::Tensor gradKey) {
    if (query.is_cuda() && key.is_cuda())
        return LaplaceKernel_backward_cuda(gradOutput, output, scale, query, key, gradQuery, gradKey);
    AT_ERROR("Not implemented on the CPU");
}

inline void LaplaceSubtraction_forward(const at::Tensor query, const at::Tensor key, at::Tensor output) {
    if (query.is_cuda() && key.is_cuda()) return LaplaceSubtraction_forward_cuda(query, key, output);
    AT_ERROR("Not implemented on the CPU");
}

inline void LaplaceSubtraction_backward_query(const at::Tensor gradOutput, const at::Tensor query,
                                              const at::Tensor key, at::Tensor gradQuery) {
    if (gradOutput.is_cuda() && query.is_cuda() && key.is_cuda())
        return LaplaceSubtraction_backward_query_cuda(gradOutput, query, key, gradQuery);
    AT_ERROR("Not implemented on the CPU");
}

inline void LaplaceSubtraction_backward_key(const at::Tensor gradOutput, const at::Tensor query,
                                            const at::Tensor key, at::Tensor gradKey) {
    if (gradOutput.is_cuda() && query.is_cuda() && key.is_cuda())
        return LaplaceSubtraction_backward_key_cuda(gradOutput, query, key, gradKey);
    AT_ERROR("Not implemented on the CPU");
}

inline void LaplaceSubtraction_reduce_forward(const at::Tensor query, const at::Tensor key, at::Tensor output) {
    if (query.is_cuda() && key.is_cuda()) return LaplaceSubtraction_reduce_forward_cuda(query, key, output);
    AT_ERROR("Not implemented on the CPU");
}

inline void LaplaceSubtraction_backward(const at::Tensor gradOutput, const at::Tensor query, const at::Tensor key,
                                        at::Tensor gradQuery, at::Tensor gradKey) {
    if (gradOutput.is_cuda() && query.is_cuda() && key.is_cuda())
        return LaplaceSubtraction_backward_cuda(gradOutput, query, key, gradQuery, gradKey);
    AT_ERROR("Not implemented on the CPU");
}

}  // namespace laplace
