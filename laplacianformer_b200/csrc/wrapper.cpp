// pybind11 module Laplace_subtraction_cuda: the reference's operator names
// and signatures (src/wrapper.cpp:73-98) plus the extended B200 operators.
#include <torch/extension.h>

#include <string>

#include "LaplaceSubtraction.h"
#include "NewtonInverse.h"
#include "laplacian_b200.h"

namespace laplace {

// "CUDA <major>.<minor>[.<patch>]" of the runtime the library was built with
// (reference src/wrapper.cpp:14-38).
std::string get_cuda_version() {
    int v = lf_cudart_version();
    std::string s = "CUDA " + std::to_string(v / 1000) + "." + std::to_string(v / 10 % 100);
    if (v % 10 != 0) s += "." + std::to_string(v % 10);
    return s;
}

bool has_cuda() { return true; }

// Host compiler of this extension (reference src/wrapper.cpp:42-69).  Built
// with std::to_string: std::ostringstream in this extension crashes at call
// time under torch 2.11 / pybind11 3 (the reference's helpers do too).
std::string get_compiler_version() {
#if defined(__clang_major__)
    return "clang " + std::to_string(__clang_major__) + "." + std::to_string(__clang_minor__) + "." +
           std::to_string(__clang_patchlevel__);
#elif defined(__GNUC__)
    return "GCC " + std::to_string(__GNUC__) + "." + std::to_string(__GNUC_MINOR__);
#else
    return "unknown";
#endif
}

}  // namespace laplace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    using namespace laplace;
    m.def("get_compiler_version", &get_compiler_version, "get_compiler_version");
    m.def("get_cuda_version", &get_cuda_version, "get_cuda_version");
    m.def("has_cuda", &has_cuda, "has_cuda");

    m.def("LaplaceSubtraction_forward", &LaplaceSubtraction_forward, "LaplaceSubtraction_forward");
    m.def("LaplaceSubtraction_backward_query", &LaplaceSubtraction_backward_query, "LaplaceSubtraction_backward_query");
    m.def("LaplaceSubtraction_backward_key", &LaplaceSubtraction_backward_key, "LaplaceSubtraction_backward_key");
    m.def("LaplaceSubtraction_reduce_forward", &LaplaceSubtraction_reduce_forward, "LaplaceSubtraction_reduce_forward");
    m.def("NewtonInverse_forward", &NewtonInverse_forward, "NewtonInverse_forward (mat, output, iter)");
    m.def("NewtonInverse_backward", &NewtonInverse_backward, "NewtonInverse_backward (grad_output, inverse, grad_mat)");
    m.def("NewtonInverse_is_supported", &NewtonInverse_is_supported, "NewtonInverse_is_supported (N)");

    // Extended operators (no counterpart in the reference module).
    m.def("LaplaceSubtraction_backward",
          [](const at::Tensor& g, const at::Tensor& q, const at::Tensor& k, c10::optional<at::Tensor> dq,
             c10::optional<at::Tensor> dk) {
              LaplaceSubtraction_backward(g, q, k, dq.has_value() ? *dq : at::Tensor(), dk.has_value() ? *dk : at::Tensor());
          },
          "LaplaceSubtraction_backward (gradOutput, query, key, gradQuery, gradKey): both gradients in one pass; "
          "pass an undefined tensor (None) to skip one",
          py::arg("gradOutput"), py::arg("query"), py::arg("key"), py::arg("gradQuery"), py::arg("gradKey"));
    m.def("LaplaceKernel_forward", &LaplaceKernel_forward,
          "LaplaceKernel_forward (query, key, output, scale): output = exp(scale * LaplaceSub(query, key)), fused",
          py::arg("query"), py::arg("key"), py::arg("output"), py::arg("scale"));
    m.def("LaplaceKernel_backward",
          [](const at::Tensor& g, const at::Tensor& out, double scale, const at::Tensor& q, const at::Tensor& k,
             c10::optional<at::Tensor> dq, c10::optional<at::Tensor> dk) {
              LaplaceKernel_backward(g, out, scale, q, k, dq.has_value() ? *dq : at::Tensor(),
                                     dk.has_value() ? *dk : at::Tensor());
          },
          "LaplaceKernel_backward (gradOutput, output, scale, query, key, gradQuery, gradKey): gradients of "
          "output = exp(scale * LaplaceSub(query, key)); dS = scale * output * gradOutput is formed in the kernel",
          py::arg("gradOutput"), py::arg("output"), py::arg("scale"), py::arg("query"), py::arg("key"),
          py::arg("gradQuery"), py::arg("gradKey"));
    m.def("NewtonInverse_forward_ex", &NewtonInverse_forward_ex,
          "NewtonInverse_forward_ex (mat, output, iter, init_mode, reg, precision)", py::arg("mat"), py::arg("output"),
          py::arg("iter"), py::arg("init_mode") = 0, py::arg("reg") = 0.01, py::arg("precision") = 0);
    m.def("NewtonInverse_residual", &NewtonInverse_residual,
          "NewtonInverse_residual (mat, inverse, residual, reg): ||(A + reg I) X - I||_F per matrix");
}
