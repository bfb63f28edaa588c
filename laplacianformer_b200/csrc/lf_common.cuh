// Shared helpers for the B200 LaplacianFormer kernels: status reporting,
// element-type traits and a few PTX wrappers.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "laplacian_b200.h"

namespace lfb {

// Records a message for lf_last_error() on the calling host thread.
void set_error(const char* fmt, ...);
void clear_error();

// Returns LF_ERR_CUDA (and records the message) when the last launch failed.
int check_launch(const char* what);

int num_sms();               // SMs of the current device (cached per device)
int max_optin_smem();        // opt-in shared memory per block (cached per device)

inline size_t dtype_size(int dtype) {
    switch (dtype) {
        case LF_F32: return 4;
        case LF_F64: return 8;
        case LF_F16: return 2;
        case LF_BF16: return 2;
        default: return 0;
    }
}

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Element traits: storage type -> accumulation type, conversions.
template <typename T> struct Elem;
template <> struct Elem<float> {
    using acc = float;
    static __device__ __forceinline__ float load(float v) { return v; }
    static __device__ __forceinline__ float store(float v) { return v; }
};
template <> struct Elem<double> {
    using acc = double;
    static __device__ __forceinline__ double load(double v) { return v; }
    static __device__ __forceinline__ double store(double v) { return v; }
};
template <> struct Elem<__half> {
    using acc = float;
    static __device__ __forceinline__ float load(__half v) { return __half2float(v); }
    static __device__ __forceinline__ __half store(float v) { return __float2half_rn(v); }
};
template <> struct Elem<__nv_bfloat16> {
    using acc = float;
    static __device__ __forceinline__ float load(__nv_bfloat16 v) { return __bfloat162float(v); }
    static __device__ __forceinline__ __nv_bfloat16 store(float v) { return __float2bfloat16_rn(v); }
};

// Dispatch a functor templated on the storage type.
#define LF_DISPATCH(dtype, T, ...)                                   \
    switch (dtype) {                                                  \
        case LF_F32: { using T = float; __VA_ARGS__; } break;         \
        case LF_F64: { using T = double; __VA_ARGS__; } break;        \
        case LF_F16: { using T = __half; __VA_ARGS__; } break;        \
        case LF_BF16: { using T = __nv_bfloat16; __VA_ARGS__; } break; \
        default: lfb::set_error("unsupported dtype code %d", dtype); return LF_ERR_DTYPE; \
    }

// Fused multiply-add in the accumulation type (explicit single/double forms,
// so that float arguments never resolve to the double-precision overload).
__device__ __forceinline__ float fma_acc(float a, float b, float c) { return __fmaf_rn(a, b, c); }
__device__ __forceinline__ double fma_acc(double a, double b, double c) { return __fma_rn(a, b, c); }

// Exact (IEEE, flush-to-zero) fp32 helpers with no contraction.
__device__ __forceinline__ float sub_ftz(float a, float b) {
    float r;
    asm("sub.rn.ftz.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float add_abs_ftz(float acc, float d) {
    // acc + |d| with one rounding; abs is a free operand modifier.
    float r, ad;
    asm("abs.ftz.f32 %0, %1;" : "=f"(ad) : "f"(d));
    asm("add.rn.ftz.f32 %0, %1, %2;" : "=f"(r) : "f"(acc), "f"(ad));
    return r;
}
// t = sat(d * 2^125 + 0.5): 1 for d > 0, 0 for d < 0, 0.5 for d == 0 (subnormal d
// flushes to zero first), so sign(d) = 2t - 1 exactly.  Overflow to +-inf
// saturates to the right end.
__device__ __forceinline__ float half_step_ftz(float d) {
    float r;
    asm("fma.rn.ftz.sat.f32 %0, %1, 0f7E000000, 0f3F000000;" : "=f"(r) : "f"(d));
    return r;
}

}  // namespace lfb
