// PyTorch-tensor front end of the Laplace_subtraction_cuda extension: argument
// checks with the reference's messages, then one call into the C ABI
// (laplacian_b200.h) on the tensor's device and current stream.  Unlike the
// reference launchers, which printf launch errors and carry on
// (src/LaplaceSubtraction_cuda_kernel.cu:481-484), every failure raises.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "LaplaceSubtraction.h"
#include "NewtonInverse.h"
#include "laplacian_b200.h"

namespace laplace {
namespace {

// Messages are assembled with std::to_string: inserting numbers into a
// std::ostream (which TORCH_CHECK does for non-string arguments) crashes at
// call time in extensions built in this image (torch 2.11, GCC 13).
std::string num(int64_t v) { return std::to_string(v); }
std::string shape_str(at::IntArrayRef s) {
    std::string r = "[";
    for (size_t i = 0; i < s.size(); ++i) r += (i ? ", " : "") + std::to_string(s[i]);
    return r + "]";
}

int dtype_code(const at::Tensor& t) {
    switch (t.scalar_type()) {
        case at::kFloat: return LF_F32;
        case at::kDouble: return LF_F64;
        case at::kHalf: return LF_F16;
        case at::kBFloat16: return LF_BF16;
        default: TORCH_CHECK(false, std::string("unsupported dtype ") + c10::toString(t.scalar_type()));
    }
    return -1;
}

lf_stream_t stream_of(const at::Tensor& t) {
    return reinterpret_cast<lf_stream_t>(at::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

void raise_on(int rc, const char* op) {
    TORCH_CHECK(rc == LF_OK, std::string(op) + " failed (code " + num(rc) + "): " + lf_last_error());
}

// Reference shape_check (src/LaplaceSubtraction_cuda.cu:12-28).
void shape_check(const at::Tensor& query, const at::Tensor& key) {
    TORCH_CHECK(query.ndimension() == 4,
                "4D weight tensor (batch size, head number, sequence length, channel) expected, but got: " +
                    num(query.ndimension()));
    TORCH_CHECK(key.ndimension() == 4,
                "4D weight tensor (batch size, head number, sequence length, channel) expected, but got: " +
                    num(key.ndimension()));
    TORCH_CHECK(query.is_contiguous(), "query tensor has to be contiguous");
    TORCH_CHECK(key.is_contiguous(), "key tensor has to be contiguous");
    TORCH_CHECK(query.size(0) == key.size(0) && query.size(1) == key.size(1) && query.size(3) == key.size(2),
                "query and key must match their size");
    TORCH_CHECK(query.scalar_type() == key.scalar_type(), "query and key must have the same dtype");
    TORCH_CHECK(query.device() == key.device(), "query and key must be on the same device");
}

void out_check(const at::Tensor& t, const at::Tensor& like, at::IntArrayRef sizes, const char* name) {
    TORCH_CHECK(t.is_cuda() && t.device() == like.device(), std::string(name) + " must be on the query's device");
    TORCH_CHECK(t.is_contiguous(), std::string(name) + " has to be contiguous");
    TORCH_CHECK(t.scalar_type() == like.scalar_type(), std::string(name) + " must have the query's dtype");
    TORCH_CHECK(t.sizes() == sizes, std::string(name) + " has shape " + shape_str(t.sizes()) + ", expected " + shape_str(sizes));
}

struct Dims {
    int64_t bh, n, m, d;
};
Dims dims_of(const at::Tensor& query, const at::Tensor& key) {
    return {query.size(0) * query.size(1), query.size(2), key.size(3), query.size(3)};
}

}  // namespace

void LaplaceSubtraction_forward_cuda(const at::Tensor query, const at::Tensor key, at::Tensor output) {
    shape_check(query, key);
    out_check(output, query, {query.size(0), query.size(1), query.size(2), key.size(3)}, "output");
    c10::cuda::CUDAGuard guard(query.device());
    Dims s = dims_of(query, key);
    raise_on(lf_laplace_sub_fwd(query.data_ptr(), key.data_ptr(), output.data_ptr(), s.bh, s.n, s.m, s.d,
                                dtype_code(query), stream_of(query)),
             "LaplaceSubtraction_forward");
}

void LaplaceKernel_forward_cuda(const at::Tensor query, const at::Tensor key, at::Tensor output, double scale) {
    shape_check(query, key);
    out_check(output, query, {query.size(0), query.size(1), query.size(2), key.size(3)}, "output");
    c10::cuda::CUDAGuard guard(query.device());
    Dims s = dims_of(query, key);
    raise_on(lf_laplace_kernel_fwd(query.data_ptr(), key.data_ptr(), output.data_ptr(), s.bh, s.n, s.m, s.d,
                                   dtype_code(query), scale, stream_of(query)),
             "LaplaceKernel_forward");
}

void LaplaceSubtraction_backward_query_cuda(const at::Tensor gradOutput, const at::Tensor query,
                                            const at::Tensor key, at::Tensor gradQuery) {
    shape_check(query, key);
    out_check(gradOutput.contiguous(), query, {query.size(0), query.size(1), query.size(2), key.size(3)}, "gradOutput");
    out_check(gradQuery, query, query.sizes(), "gradQuery");
    c10::cuda::CUDAGuard guard(query.device());
    at::Tensor g = gradOutput.contiguous();
    Dims s = dims_of(query, key);
    raise_on(lf_laplace_sub_bwd_query(g.data_ptr(), query.data_ptr(), key.data_ptr(), gradQuery.data_ptr(), s.bh,
                                      s.n, s.m, s.d, dtype_code(query), stream_of(query)),
             "LaplaceSubtraction_backward_query");
}

void LaplaceSubtraction_backward_key_cuda(const at::Tensor gradOutput, const at::Tensor query, const at::Tensor key,
                                          at::Tensor gradKey) {
    shape_check(query, key);
    out_check(gradOutput.contiguous(), query, {query.size(0), query.size(1), query.size(2), key.size(3)}, "gradOutput");
    out_check(gradKey, query, key.sizes(), "gradKey");
    c10::cuda::CUDAGuard guard(query.device());
    at::Tensor g = gradOutput.contiguous();
    Dims s = dims_of(query, key);
    raise_on(lf_laplace_sub_bwd_key(g.data_ptr(), query.data_ptr(), key.data_ptr(), gradKey.data_ptr(), s.bh, s.n,
                                    s.m, s.d, dtype_code(query), stream_of(query)),
             "LaplaceSubtraction_backward_key");
}

void LaplaceSubtraction_backward_cuda(const at::Tensor gradOutput, const at::Tensor query, const at::Tensor key,
                                      at::Tensor gradQuery, at::Tensor gradKey) {
    shape_check(query, key);
    out_check(gradOutput.contiguous(), query, {query.size(0), query.size(1), query.size(2), key.size(3)}, "gradOutput");
    if (gradQuery.defined()) out_check(gradQuery, query, query.sizes(), "gradQuery");
    if (gradKey.defined()) out_check(gradKey, query, key.sizes(), "gradKey");
    c10::cuda::CUDAGuard guard(query.device());
    at::Tensor g = gradOutput.contiguous();
    Dims s = dims_of(query, key);
    if (gradQuery.defined() && gradKey.defined()) {
        // Balanced kernel when the shape has one: its workspace comes from
        // the caching allocator on the op's stream.
        const size_t need = lf_laplace_sub_bwd_workspace_size(s.bh, s.n, s.m, s.d, dtype_code(query));
        if (need) {
            at::Tensor ws = at::empty({(int64_t)need}, query.options().dtype(at::kByte));
            raise_on(lf_laplace_sub_bwd_ws(g.data_ptr(), query.data_ptr(), key.data_ptr(), gradQuery.data_ptr(),
                                           gradKey.data_ptr(), s.bh, s.n, s.m, s.d, dtype_code(query), ws.data_ptr(),
                                           need, stream_of(query)),
                     "LaplaceSubtraction_backward");
            return;
        }
    }
    raise_on(lf_laplace_sub_bwd(g.data_ptr(), query.data_ptr(), key.data_ptr(),
                                gradQuery.defined() ? gradQuery.data_ptr() : nullptr,
                                gradKey.defined() ? gradKey.data_ptr() : nullptr, s.bh, s.n, s.m, s.d,
                                dtype_code(query), stream_of(query)),
             "LaplaceSubtraction_backward");
}

void LaplaceKernel_backward_cuda(const at::Tensor gradOutput, const at::Tensor output, double scale,
                                 const at::Tensor query, const at::Tensor key, at::Tensor gradQuery,
                                 at::Tensor gradKey) {
    shape_check(query, key);
    const std::vector<int64_t> sshape = {query.size(0), query.size(1), query.size(2), key.size(3)};
    out_check(gradOutput.contiguous(), query, sshape, "gradOutput");
    out_check(output, query, sshape, "output");
    if (gradQuery.defined()) out_check(gradQuery, query, query.sizes(), "gradQuery");
    if (gradKey.defined()) out_check(gradKey, query, key.sizes(), "gradKey");
    c10::cuda::CUDAGuard guard(query.device());
    at::Tensor g = gradOutput.contiguous();
    Dims s = dims_of(query, key);
    at::Tensor ws;
    size_t need = 0;
    if (gradQuery.defined() && gradKey.defined()) {
        need = lf_laplace_sub_bwd_workspace_size(s.bh, s.n, s.m, s.d, dtype_code(query));
        if (need) ws = at::empty({(int64_t)need}, query.options().dtype(at::kByte));
    }
    raise_on(lf_laplace_kernel_bwd(g.data_ptr(), output.data_ptr(), query.data_ptr(), key.data_ptr(),
                                   gradQuery.defined() ? gradQuery.data_ptr() : nullptr,
                                   gradKey.defined() ? gradKey.data_ptr() : nullptr, s.bh, s.n, s.m, s.d,
                                   dtype_code(query), scale, need ? ws.data_ptr() : nullptr, need,
                                   stream_of(query)),
             "LaplaceKernel_backward");
}

void LaplaceSubtraction_reduce_forward_cuda(const at::Tensor query, const at::Tensor key, at::Tensor output) {
    shape_check(query, key);
    out_check(output, query, {query.size(0), query.size(1), query.size(2), key.size(3)}, "output");
    c10::cuda::CUDAGuard guard(query.device());
    Dims s = dims_of(query, key);
    raise_on(lf_laplace_sub_reduce_fwd(query.data_ptr(), key.data_ptr(), output.data_ptr(), s.bh, s.n, s.m, s.d,
                                       dtype_code(query), stream_of(query)),
             "LaplaceSubtraction_reduce_forward");
}

bool NewtonInverse_supports(int N) { return lf_newton_inverse_supported(N) != 0; }

// Reference NewtonInverse_forward_cuda checks (src/NewtonInverse_cuda_kernel.cu:764-779).
static void ns_checks(const at::Tensor& mat, const at::Tensor& output) {
    TORCH_CHECK(mat.is_contiguous(), "mat must be contiguous");
    TORCH_CHECK(output.is_contiguous(), "output must be contiguous");
    TORCH_CHECK(mat.sizes() == output.sizes(), "mat and output must have the same shape");
    TORCH_CHECK(output.is_cuda() && output.device() == mat.device(), "output must be on mat's device");
    TORCH_CHECK(output.scalar_type() == mat.scalar_type(), "output must have mat's dtype");
    const int64_t N = mat.size(2);
    TORCH_CHECK(NewtonInverse_supports((int)N), "NewtonInverse: N=" + num(N) +
                " is not supported on this device (insufficient smem or out of range)");
}

void NewtonInverse_forward_ex_cuda(const at::Tensor mat, at::Tensor output, int iter, int init_mode, double reg,
                                   int precision) {
    ns_checks(mat, output);
    c10::cuda::CUDAGuard guard(mat.device());
    raise_on(lf_newton_inverse_fwd_ex(mat.data_ptr(), output.data_ptr(), mat.size(0) * mat.size(1), mat.size(2), iter,
                                      dtype_code(mat), init_mode, reg, precision, stream_of(mat)),
             "NewtonInverse_forward");
}

void NewtonInverse_forward_cuda(const at::Tensor mat, at::Tensor output, int iter) {
    NewtonInverse_forward_ex_cuda(mat, output, iter, LF_NS_INIT_REFERENCE, 0.01, LF_NS_PREC_SPLIT3);
}

void NewtonInverse_backward_cuda(const at::Tensor grad_output, const at::Tensor inverse, at::Tensor grad_mat) {
    c10::cuda::CUDAGuard guard(inverse.device());
    TORCH_CHECK(grad_output.is_contiguous(), "grad_output must be contiguous");
    TORCH_CHECK(inverse.is_contiguous(), "inverse must be contiguous");
    TORCH_CHECK(grad_mat.is_contiguous(), "grad_mat must be contiguous");
    TORCH_CHECK(grad_output.sizes() == inverse.sizes() && inverse.sizes() == grad_mat.sizes(), "shape mismatch");
    TORCH_CHECK(grad_output.scalar_type() == inverse.scalar_type() && grad_mat.scalar_type() == inverse.scalar_type(),
                "dtype mismatch");
    TORCH_CHECK(grad_mat.is_cuda() && grad_mat.device() == inverse.device(), "grad_mat must be on inverse's device");
    const int64_t N = inverse.size(2);
    TORCH_CHECK(inverse.size(3) == N, "last two dims must be equal");
    TORCH_CHECK(NewtonInverse_supports((int)N), "NewtonInverse: N=" + num(N) +
                " is not supported on this device (insufficient smem or out of range)");
    raise_on(lf_newton_inverse_bwd(grad_output.data_ptr(), inverse.data_ptr(), grad_mat.data_ptr(),
                                   inverse.size(0) * inverse.size(1), N, dtype_code(inverse), stream_of(inverse)),
             "NewtonInverse_backward");
}

void NewtonInverse_residual_cuda(const at::Tensor mat, const at::Tensor inverse, at::Tensor residual, double reg) {
    c10::cuda::CUDAGuard guard(mat.device());
    TORCH_CHECK(mat.dim() == 4 && mat.size(2) == mat.size(3), "mat must be (B,H,N,N)");
    TORCH_CHECK(mat.is_contiguous() && inverse.is_contiguous() && residual.is_contiguous(), "tensors must be contiguous");
    TORCH_CHECK(mat.sizes() == inverse.sizes() && mat.scalar_type() == inverse.scalar_type(), "mat/inverse mismatch");
    TORCH_CHECK(residual.numel() == mat.size(0) * mat.size(1), "residual must have B*H elements");
    TORCH_CHECK(residual.scalar_type() == (mat.scalar_type() == at::kDouble ? at::kDouble : at::kFloat),
                "residual must be float32 (float64 for float64 input)");
    raise_on(lf_newton_inverse_residual(mat.data_ptr(), inverse.data_ptr(), residual.data_ptr(),
                                        mat.size(0) * mat.size(1), mat.size(2), reg, dtype_code(mat), stream_of(mat)),
             "NewtonInverse_residual");
}

}  // namespace laplace
