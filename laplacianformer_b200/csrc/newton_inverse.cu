// NewtonInverse on B200 (sm_100a): batched Newton–Schulz inverse of small
// square matrices and its analytic backward.
//
// Semantics follow src/NewtonInverse_cuda_kernel.cu of the reference:
//   P = A + reg*I (reg = 0.01, :169), alpha = 1.8 / (max_i sum_j P_ij)^2
//   (:82-120), V0 = alpha*P (:176-178), then `iters` times V <- 2V - V P V
//   (:181-248 / :381-457); backward dA = -(V^T G V^T) (:469-573).
// An extended initialisation X0 = P^T / (||P||_1 ||P||_inf) is also offered.
//
// Tensor-core path (fp32 / fp16 / bf16 inputs, n <= 128), one CTA per matrix:
// * The matrix is zero padded to 128x128.  Every product runs on tcgen05 as
//   kind::f16 MMAs (M = N = 128, K = 16) with fp32 accumulation in tensor
//   memory.  Each fp32 operand X is split as X*s = hi + lo with hi, lo fp16
//   and s a power of two that puts max|X*s| in [2^14, 2^15); the product is
//   hi_a*hi_b + hi_a*lo_b + lo_a*hi_b (the lo*lo term is below 2^-22 of the
//   result), i.e. about 22 significant bits — the same accuracy class as the
//   reference's fp32 CUDA-core loops at twice the rate of a 3xTF32 split and
//   with half its shared-memory footprint.
// * P, V and W = V P are kept in shared memory as hi/lo fp16 in the 128-byte
//   swizzled row-major layout; the same bytes serve as a K-major A operand
//   and as an MN-major B operand, so no transposed copies are needed:
//       W = V P  (A = V, B = P),   Y = W V  (A = W, B = V),   V <- 2V - Y.
//   This is the association of the reference's 2-buffer kernel (:389-456).
// * The exact fp32 V lives in tensor memory next to the accumulator (256
//   columns in total), so the update 2V - Y is done in fp32.
// * One elected thread issues the MMAs and commits them to an mbarrier; all
//   waits are bounded and report LF_ERR_TIMEOUT through a device status word
//   instead of hanging.
//
// CUDA-core path: fp64 inputs, the LF_NS_PREC_FP32_SIMT mode, the backward
// and the residual use row-blocked fp32/fp64 FMA loops with V resident in
// shared memory.
#include <cooperative_groups.h>

#include "lf_common.cuh"

namespace cg = cooperative_groups;

namespace lfb {

// Device status word: 0 = ok, otherwise an lf_status code set by a kernel
// whose bounded wait expired.  Read and cleared by lf_device_status().
__device__ int g_ns_status = 0;

int peer_status(bool clear);  // peer.cu

namespace {

constexpr int kTcThreads = 256;            // 8 warps; two CTAs share an SM
constexpr int kTile = 128;                 // padded matrix size (one tile)
constexpr int kOpBytes = kTile * kTile * 2; // one fp16 operand (32 KB)
constexpr int kTmemCols = 256;             // accumulator [0,128), P hi [128,192), P lo [192,256)
constexpr int kLtChunk = 64;               // landmark channels staged per set-up pass

// Matrices per 128x128 tile: floor(128/n) for n <= 64 (block-diagonal), else 1.
int tc_per_tile(int64_t n) { return n <= kTile / 2 ? (int)(kTile / n) : 1; }

// ---------------------------------------------------------------------------
// PTX wrappers (tcgen05, mbarrier, fences)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Returns true when the phase with the given parity has completed, false if
// it has not completed within about two seconds (bounded wait; the caller
// reports LF_ERR_TIMEOUT instead of hanging the GPU).  Each try_wait may
// suspend the thread for up to 20 us until the phase completes, so waiting
// warps do not spin on the issue slots the epilogue warps need.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns = 2000000000ull) {
    const uint32_t addr = smem_u32(bar);
    uint64_t t0 = 0;
    for (uint32_t spin = 0;; ++spin) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}\n"
            : "=r"(done)
            : "r"(addr), "r"(parity), "r"(20000u)
            : "memory");
        if (done) return true;
        if (spin == 0) t0 = global_ns();
        else if (global_ns() - t0 > limit_ns) return false;
    }
}

// One lane of the calling (converged) warp returns true.
__device__ __forceinline__ bool elect_one() {
    uint32_t pred;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "elect.sync _|p, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(pred));
    return pred != 0;
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic: one issue slot per pair).
__device__ __forceinline__ uint64_t pk2(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void upk2(uint64_t v, float& a, float& b) { asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v)); }
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
// fp16 pair of (lo, hi) = the two floats of v (first float in the low half).
__device__ __forceinline__ __half2 cvt_h2(uint64_t v) {
    float a, b;
    upk2(v, a, b);
    return __float22half2_rn(make_float2(a, b));
}
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<const uint32_t*>(&h); }

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem] (+)= A[smem] * B[smem], kind::f16, cta_group::1, issued by the
// lane with go != 0.  The whole warp executes the instruction (predicated),
// so descriptors computed in converged code stay in uniform registers and
// each MMA issues in a few cycles; an MMA inside a one-lane branch measured
// about twice the tensor pipe's time per instruction.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate, uint32_t go) {
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "setp.ne.b32 q, %5, 0;\n\t"
        "@q tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(go)
        : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem], kind::f16: A is 128 lanes (rows) x K fp16
// with consecutive K pairs packed in one 32-bit column (lower K in the low half).
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate, uint32_t go) {
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "setp.ne.b32 q, %5, 0;\n\t"
        "@q tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(go)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns: thread i of the warp gets lane
// (quadrant*32 + i), columns [col, col+16).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t* r = reinterpret_cast<uint32_t*>(v);
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
// 32 lanes x 8 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t* r = reinterpret_cast<uint32_t*>(v);
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// Ties registers written by tcgen05.ld to a point after tcgen05.wait::ld so
// that the compiler cannot hoist their uses above the wait.
template <int N>
__device__ __forceinline__ void reg_fence(float (&v)[N]) {
#pragma unroll
    for (int i = 0; i < N; ++i) asm volatile("" : "+f"(v[i]));
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------------------
// Operand layout: a 128x128 fp16 matrix X[r][c], row-major with the 128-byte
// swizzle.  Columns [0,64) and [64,128) form two 16 KB blocks; row r of a
// block is 128 bytes at r*128 and its 16-byte chunk k (columns 8k..8k+7 of
// the block) sits at chunk k^(r%8).  The same bytes are a K-major A operand
// and an MN-major B operand.
// ---------------------------------------------------------------------------

// Shared-memory matrix descriptor (sm_100): start>>4 [0,14), LBO>>4 [16,30),
// SBO>>4 [32,46), version 1 at bit 46, layout SWIZZLE_128B (2) at [61,64).
__device__ __forceinline__ uint64_t make_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}
// kind::f16 instruction descriptor: fp32 accumulator, fp16 A and B, A
// K-major, B MN-major, N = M = 128.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 16) | ((uint32_t)(kTile >> 3) << 17) | ((uint32_t)(kTile >> 4) << 24);

// Power-of-two scale that maps max|x| into [2^14, 2^15); 1 for 0, negative
// or non-finite input, 2^127 for subnormal input.  Built from the exponent
// bits: a handful of integer instructions on the epilogues' critical path.
__device__ __forceinline__ float split_scale(float mx) {
    const uint32_t b = __float_as_uint(mx);
    const int e = (int)((b >> 23) & 0xffu);  // biased exponent: mx in [2^(e-127), 2^(e-126))
    if (!(mx > 0.f) || e == 0xff) return 1.f;
    const int se = min(127 + 141 - e, 254);  // s = 2^(14 - (e - 127))
    return __uint_as_float((uint32_t)se << 23);
}

__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// Row `r`, 64 columns of V * s into the operand buffers (vh_row: shared
// address of the row's 64-column block in V hi; V lo follows V hi at
// kOpBytes): hi always, lo = fp16(V*s - hi) when `lo` (16-byte swizzled
// chunks, conflict-free across the 32 rows of a warp).  Returns max|hi|
// (= max|V| s up to the fp16 rounding of hi).
__device__ __forceinline__ float store_v(uint32_t vh_row, int rx, const float (&v)[64], float s, bool lo) {
    const uint64_t ss = pk2(s, s);
    __half2 hm0 = __float2half2_rn(0.f), hm1 = hm0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        uint32_t h[4], l[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const uint64_t xs = mul2(pk2(v[8 * k + 2 * e], v[8 * k + 2 * e + 1]), ss);
            const __half2 hh = cvt_h2(xs);
            if (e & 1) hm1 = __hmax2(hm1, __habs2(hh));
            else hm0 = __hmax2(hm0, __habs2(hh));
            h[e] = h2u(hh);
            if (lo) {
                const float2 hb = __half22float2(hh);
                l[e] = h2u(cvt_h2(sub2(xs, pk2(hb.x, hb.y))));
            }
        }
        const uint32_t off = vh_row + ((k ^ rx) << 4);
        sts128(off, h[0], h[1], h[2], h[3]);
        if (lo) sts128(off + kOpBytes, l[0], l[1], l[2], l[3]);
    }
    const __half2 hm = __hmax2(hm0, hm1);
    return fmaxf(__low2float(hm), __high2float(hm));
}

// G * sG for 16 accumulator columns (chunk j16 of the thread's 64) holding
// H * sP * sV, stored as fp16 into the G operand: g = delta - H, so the scaled
// value is acc * chs (+ sG on the diagonal) with chs = -sG/(sP sV).
// DIAG: column j of the chunk is the diagonal for the lane with lane == j + joff.
template <bool DIAG>
__device__ __forceinline__ void g_store(const float (&a)[16], uint64_t chs2, float sG, int lane, int joff,
                                        __half2& hm, uint32_t gh_row, int rx, int j16) {
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        uint32_t hp[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int j = 8 * q + 2 * e;
            uint64_t g;
            if (DIAG) g = fma2(pk2(a[j], a[j + 1]), chs2, pk2((j + joff == lane) ? sG : 0.f, (j + 1 + joff == lane) ? sG : 0.f));
            else g = mul2(pk2(a[j], a[j + 1]), chs2);
            const __half2 h = cvt_h2(g);
            hm = __hmax2(hm, __habs2(h));
            hp[e] = h2u(h);
        }
        sts128(gh_row + (((2 * j16 + q) ^ rx) << 4), hp[0], hp[1], hp[2], hp[3]);
    }
}

// fp16 hi (lo = false) or lo (lo = true) part of 16 values times s, packed
// in pairs (element 2i in the low half).
__device__ __forceinline__ void split_half(const float (&v)[16], float s, bool lo, uint32_t (&out)[8]) {
    const uint64_t ss = pk2(s, s);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const uint64_t xs = mul2(pk2(v[2 * e], v[2 * e + 1]), ss);
        __half2 hh = cvt_h2(xs);
        if (lo) {
            const float2 hb = __half22float2(hh);
            hh = cvt_h2(sub2(xs, pk2(hb.x, hb.y)));
        }
        out[e] = h2u(hh);
    }
}

// Max over the lanes of this warp that hold rows of the same matrix (the
// rows of one matrix are consecutive lanes); bit i of `seg` is set when lane
// + 2^i holds a row of the same matrix.  The matrix's first lane in the warp
// ends with the warp's maximum.
__device__ __forceinline__ float seg_max(float v, uint32_t seg) {
#pragma unroll
    for (int i = 0; i < 5; ++i) {
        const float w = __shfl_down_sync(0xffffffffu, v, 1 << i);
        if (seg & (1u << i)) v = fmaxf(v, w);
    }
    return v;
}

// seg_max for non-negative values; when one matrix owns all 32 rows of the
// warp (`warp_one`) it is a single warp-wide integer max of the float bits.
__device__ __forceinline__ float seg_max_nn(float v, uint32_t seg, bool warp_one) {
    if (warp_one) return __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(v)));
    return seg_max(v, seg);
}

// Order-preserving map of floats to unsigned ints (for atomicMax on signed values).
__device__ __forceinline__ uint32_t ord_bits(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ord_float(uint32_t u) {
    return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

struct NsShared {
    uint64_t bar[2];          // [0]: H = P V complete, [1]: Y = V G complete
    uint32_t tmem_base;
    uint32_t gmax[2][kTile];  // per matrix of the tile: max|G * sG| (float bits), by iteration parity
    uint32_t vmax[2][kTile];  // per matrix: max|V| (float bits), by iteration parity
    uint32_t stat[4][kTile];  // set-up: max signed row sum (ordered bits), max |row| sum, max |column| sum, max|P|
    float part[2][kTile][4];  // set-up: the two column halves' row sum, |row| sum, max|P| and |column| sum
};

// Set-up staging tile: 128x128 fp32, 16-byte chunk c/4 of row i at chunk
// (c/4) ^ (i%32).  Float4 row accesses by lanes over rows or over chunks,
// and scalar column reads by lanes over columns or rows, are conflict-free.
__device__ __forceinline__ int stage_idx(int i, int c) { return i * kTile + ((((c >> 2) ^ i) & 31) << 2) + (c & 3); }
__device__ __forceinline__ float4 stage_ld4(const float* st, int i, int c4) {
    return *reinterpret_cast<const float4*>(st + i * kTile + (((c4 ^ i) & 31) << 2));
}
__device__ __forceinline__ void stage_st4(float* st, int i, int c4, float4 v) {
    *reinterpret_cast<float4*>(st + i * kTile + (((c4 ^ i) & 31) << 2)) = v;
}

// Row `row`, columns [c0, c0+64) of the iterate to the output (columns of
// the row's own matrix only).  xr points at the row's first element.
template <typename T>
__device__ __forceinline__ void store_rows(T* __restrict__ xr, int c0, int bn, int n, const float (&v)[64]) {
    if constexpr (sizeof(T) == 4) {
        if (n == kTile && (reinterpret_cast<uintptr_t>(xr + c0) & 15) == 0) {
#pragma unroll
            for (int j = 0; j < 64; j += 4)
                *reinterpret_cast<float4*>(xr + c0 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            return;
        }
    }
#pragma unroll
    for (int j = 0; j < 64; ++j) {
        const int c = c0 + j - bn;
        if ((unsigned)c < (unsigned)n) xr[c] = Elem<T>::store(v[j]);
    }
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
                 "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}

// H (+)= P V with A = P from tensor memory (hi at a_phi, lo at a_plo) and B =
// V from shared memory (descriptors of K step 0; a K step of 16 rows is 2 KB,
// 128 in the descriptor's address field).  FULL adds P_hi V_lo + P_lo V_hi.
template <bool FULL>
__device__ __forceinline__ void issue_h(uint32_t acc, uint32_t a_phi, uint32_t a_plo, uint64_t dvh, uint64_t dvl,
                                        uint32_t go) {
#pragma unroll
    for (int ks = 0; ks < kTile / 16; ++ks) {
        mma_f16_ts(acc, a_phi + ks * 8, dvh + (uint64_t)(ks * 128), kIdesc, ks > 0 ? 1u : 0u, go);
        if (FULL) {
            mma_f16_ts(acc, a_phi + ks * 8, dvl + (uint64_t)(ks * 128), kIdesc, 1u, go);
            mma_f16_ts(acc, a_plo + ks * 8, dvh + (uint64_t)(ks * 128), kIdesc, 1u, go);
        }
    }
}

// Y (+)= V G with A = V (K-major view; a K step is 32 bytes within a 64-column
// block of 16 KB) and B = G (MN-major), both in shared memory.  FULL adds V_lo G.
template <bool FULL>
__device__ __forceinline__ void issue_y(uint32_t acc, uint64_t dah, uint64_t dal, uint64_t dg, uint32_t go) {
#pragma unroll
    for (int ks = 0; ks < kTile / 16; ++ks) {
        const uint64_t ao = (uint64_t)((ks >> 2) * 1024 + (ks & 3) * 2);
        mma_f16(acc, dah + ao, dg + (uint64_t)(ks * 128), kIdesc, ks > 0 ? 1u : 0u, go);
        if (FULL) mma_f16(acc, dal + ao, dg + (uint64_t)(ks * 128), kIdesc, 1u, go);
    }
}

// Newton–Schulz on tcgen05 tensor cores, in the residual form
//     H = P V,  G = I - H,  V <- V + V G        (= 2V - V P V)
// One CTA per 128x128 tile; for n <= 64 a tile holds floor(128/n) matrices
// on its diagonal (products of block-diagonal matrices stay block-diagonal,
// every scale is per matrix).  Two CTAs share an SM, so one CTA's epilogues
// run while the other's products occupy the tensor pipe.
//
// Storage per CTA: P (hi, lo fp16) as the A operand in tensor memory next to
// the fp32 accumulator (256 columns); V hi/lo and G hi in shared memory
// (96 KB, 128-byte swizzle, used as MN-major B and K-major A operands); the
// exact fp32 V in registers (thread = row, 64 columns).
// Per iteration (one elected lane of warp 0 issues the MMAs):
//   H   = P_hi V_hi [+ P_hi V_lo + P_lo V_hi]     A from tensor memory
//   G*sG = fp16((delta - H) sG)                   scale from max|G| <= 1 + ||P||_inf max|V|
//   Y   = V_hi G_hi [+ V_lo G_hi]                 A and B from shared memory
//   V  += Y;  V hi/lo with a scale from max|V'| <= max|V| (1 + n max|G|)
// The bracketed terms run on "full" iterations (every iteration for split3,
// the last two for mixed).  The V correction Y is scaled by |G|, which goes
// to zero as the iteration converges, so a single fp16 G suffices; its V
// factor needs hi + lo so that V's own rounding does not enter the residual.
// max|G| and max|V| are reduced across the tile piggybacking on the two
// barriers that hand the operands to the MMA thread.
template <typename T>
__global__ void __launch_bounds__(kTcThreads, 2)
ns_tc_fwd_kernel(const T* __restrict__ a, T* __restrict__ x, int batch, int n, int nb, int iters, int mode,
                 float reg, int precision, const float* __restrict__ lmk, int ld, float lscale, int pf_ahead) {
    extern __shared__ __align__(16) unsigned char smem_raw[];  // re-aligned to 1024 below
    // V hi at [0, 32K), V lo at [32K, 64K), G hi at [64K, 96K) of the aligned
    // base; addresses are recomputed from the base where they are used, so
    // no pointer has to stay live across the iteration loop.
    unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* stage = reinterpret_cast<float*>(base + kOpBytes);  // set-up: 128x128 fp32 over V lo and G hi
    float* LT = reinterpret_cast<float*>(base);                // landmark set-up: [kLtChunk][128] fp32
    NsShared& sh = *reinterpret_cast<NsShared*>(base + 3 * kOpBytes);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quad = warp & 3, half = warp >> 2;
    const int row = quad * 32 + lane;  // tile row (= TMEM lane) this thread owns
    const int c0 = half * 64;          // its 64 columns
    const uint32_t rbase = (uint32_t)(half * 16384 + row * 128);  // its row in a fp16 operand
    const int rx = row & 7;
    const int64_t m0 = (int64_t)blockIdx.x * nb;
    const int nrows = (int)min((int64_t)nb, (int64_t)batch - m0) * n;
    const bool valid = row < nrows;
    const int blk = valid ? row / n : -1;  // matrix of the tile that owns this row
    const int bn = valid ? blk * n : 0;
    // which of the thread's two 32-column chunks holds its diagonal (warp-uniform)
    const int dchunk = ((quad >> 1) == half) ? (quad & 1) : -1;

    if (tid == 0) {
        mbar_init(&sh.bar[0], 1);
        mbar_init(&sh.bar[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int e = tid; e < kTile; e += kTcThreads) {
        sh.gmax[0][e] = sh.gmax[1][e] = sh.vmax[0][e] = sh.vmax[1][e] = 0u;
        sh.stat[0][e] = sh.stat[1][e] = sh.stat[2][e] = sh.stat[3][e] = 0u;
    }
    if (warp == 0) tmem_alloc(&sh.tmem_base, kTmemCols);
    uint32_t seg = 0;
#pragma unroll
    for (int i = 0; i < 5; ++i) {
        const int o = __shfl_down_sync(0xffffffffu, blk, 1 << i);
        if (valid && lane + (1 << i) < 32 && o == blk) seg |= 1u << i;
    }
    const int prev = __shfl_up_sync(0xffffffffu, blk, 1);
    const bool leader = valid && (lane == 0 || prev != blk);
    // (the shuffle runs on every lane: it must not sit behind the `valid &&`)
    const int blk0 = __shfl_sync(0xffffffffu, blk, 0);
    const bool warp_one = __all_sync(0xffffffffu, valid && blk == blk0);

    // ---- set-up: P = A + reg I into the staging tile ------------------------
    if (lmk) {
        // A[i][c] = exp(lscale * sum_k |L[i][k] - L[c][k]|), channel sums in
        // order with the LaplaceSub forward's fp32 operations, so A is
        // bit-identical to lf_laplace_kernel_fwd(L, L^T).
        float acc[64];
#pragma unroll
        for (int j = 0; j < 64; ++j) acc[j] = 0.f;
        for (int k0 = 0; k0 < ld; k0 += kLtChunk) {
            const int kc = min(kLtChunk, ld - k0);
            __syncthreads();  // the previous chunk has been consumed
            {
                const int i = tid & (kTile - 1);
                const bool iv = i < nrows;
                const float* Lr = lmk + (iv ? ((m0 + i / n) * (int64_t)n + i % n) * ld + k0 : 0);
                for (int kk = tid >> 7; kk < kc; kk += kTcThreads / kTile) LT[kk * kTile + i] = iv ? Lr[kk] : 0.f;
            }
            __syncthreads();
            if (valid) {
                for (int kk = 0; kk < kc; ++kk) {
                    const float li = LT[kk * kTile + row];
                    const float4* lc = reinterpret_cast<const float4*>(LT + kk * kTile + c0);
#pragma unroll
                    for (int j4 = 0; j4 < 16; ++j4) {
                        const float4 w = lc[j4];
                        acc[4 * j4 + 0] = add_abs_ftz(acc[4 * j4 + 0], sub_ftz(li, w.x));
                        acc[4 * j4 + 1] = add_abs_ftz(acc[4 * j4 + 1], sub_ftz(li, w.y));
                        acc[4 * j4 + 2] = add_abs_ftz(acc[4 * j4 + 2], sub_ftz(li, w.z));
                        acc[4 * j4 + 3] = add_abs_ftz(acc[4 * j4 + 3], sub_ftz(li, w.w));
                    }
                }
            }
        }
#pragma unroll
        for (int j4 = 0; j4 < 16; ++j4) {
            float t[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int c = c0 + 4 * j4 + q;
                t[q] = 0.f;
                if (valid && (unsigned)(c - bn) < (unsigned)n) t[q] = expf(lscale * acc[4 * j4 + q]) + (c == row ? reg : 0.f);
            }
            stage_st4(stage, row, (c0 >> 2) + j4, make_float4(t[0], t[1], t[2], t[3]));
        }
    } else {
        // Gather: warp w covers tile rows w, w+8, ...; lane l columns 4l..4l+3.
        const T* A = a + m0 * (int64_t)n * n;
        if (tid == 0 && pf_ahead > 0 && (int64_t)blockIdx.x + pf_ahead < (int64_t)gridDim.x) {
            // Warm L2 with the tile of the CTA that follows `pf_ahead` slots
            // later (the next wave): its gather then reads L2, not HBM.
            const int64_t t = (int64_t)blockIdx.x + pf_ahead;
            const int64_t mt = min((int64_t)nb, (int64_t)batch - t * nb);
            const uintptr_t lo = (reinterpret_cast<uintptr_t>(a + t * nb * (int64_t)n * n) + 15) & ~uintptr_t(15);
            const uintptr_t hi = reinterpret_cast<uintptr_t>(a + (t * nb + mt) * (int64_t)n * n) & ~uintptr_t(15);
            for (uintptr_t p = lo; p < hi; p += 32768) {
                const uint32_t sz = (uint32_t)min((uintptr_t)32768, hi - p);
                asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(sz) : "memory");
            }
        }
        bool whole = false;  // fp32, n = 128, 16-byte aligned rows: 16 row loads in flight per thread
        if constexpr (sizeof(T) == 4) whole = n == kTile && (reinterpret_cast<uintptr_t>(A) & 15) == 0;
        if (whole) {
            float4 v[kTile / 8];
#pragma unroll
            for (int it = 0; it < kTile / 8; ++it)
                v[it] = __ldg(reinterpret_cast<const float4*>(A + (int64_t)(warp + 8 * it) * kTile) + lane);
#pragma unroll
            for (int it = 0; it < kTile / 8; ++it) {
                const int i = warp + 8 * it;
                float4 w = v[it];
                if ((i >> 2) == lane) {  // the diagonal: column i = component i & 3 (= warp & 3) of lane i / 4
                    const int q = warp & 3;
                    w.x += q == 0 ? reg : 0.f;
                    w.y += q == 1 ? reg : 0.f;
                    w.z += q == 2 ? reg : 0.f;
                    w.w += q == 3 ? reg : 0.f;
                }
                stage_st4(stage, i, lane, w);
            }
        }
        int b = warp / n, r = warp - (warp / n) * n;  // matrix and row within it of tile row `warp`
#pragma unroll 4
        for (int it = 0; it < (whole ? 0 : kTile / 8); ++it) {
            const int i = warp + 8 * it;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (i < nrows) {
                const int ib = b * n;
                const T* Ar = A + ((int64_t)b * n + r) * n - ib;  // Ar[c] for c in [ib, ib+n)
                bool done = false;
                if constexpr (sizeof(T) == 4) {
                    if (n == kTile && (reinterpret_cast<uintptr_t>(Ar + 4 * lane) & 15) == 0) {
                        v = *reinterpret_cast<const float4*>(Ar + 4 * lane);
                        done = true;
                    }
                }
                if (!done) {
                    float* vp = &v.x;
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        if ((unsigned)(4 * lane + q - ib) < (unsigned)n) vp[q] = Elem<T>::load(Ar[4 * lane + q]);
                }
                if ((i >> 2) == lane) (&v.x)[i & 3] += reg;
            }
            stage_st4(stage, i, lane, v);
            r += 8;
            while (r >= n) { r -= n; ++b; }
        }
    }
    __syncthreads();

    // ---- per-matrix statistics (rows and columns of the tile are the
    // thread's `row` index; the two column halves meet in shared memory) ------
    // Column |.| sums: warp w adds tile rows w, w+8, ... of lane l's columns
    // 4l..4l+3 into colp[w] (in the V hi region, free until V0 is stored);
    // the eight partials are added in warp order below.  The same order for
    // every input path, so the landmark-fused form stays bit-identical.
    float* colp = reinterpret_cast<float*>(base);  // [8][kTile]
    {
        float rs = 0.f, ra = 0.f, pm = 0.f;
#pragma unroll 4
        for (int c4 = 0; c4 < 16; ++c4) {
            const float4 p = stage_ld4(stage, row, 16 * half + c4);
            rs += (p.x + p.y) + (p.z + p.w);
            ra += (fabsf(p.x) + fabsf(p.y)) + (fabsf(p.z) + fabsf(p.w));
            pm = fmaxf(pm, fmaxf(fmaxf(fabsf(p.x), fabsf(p.y)), fmaxf(fabsf(p.z), fabsf(p.w))));
        }
        float4 cp = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
        for (int it = 0; it < kTile / 8; ++it) {
            const float4 p = stage_ld4(stage, warp + 8 * it, lane);
            cp.x += fabsf(p.x); cp.y += fabsf(p.y); cp.z += fabsf(p.z); cp.w += fabsf(p.w);
        }
        *reinterpret_cast<float4*>(colp + warp * kTile + 4 * lane) = cp;
        sh.part[half][row][0] = rs;
        sh.part[half][row][1] = ra;
        sh.part[half][row][2] = pm;
    }
    __syncthreads();
    {
        float rs = sh.part[0][row][0] + sh.part[1][row][0];
        float ra = sh.part[0][row][1] + sh.part[1][row][1];
        float pm = fmaxf(sh.part[0][row][2], sh.part[1][row][2]);
        float cs = colp[row];
#pragma unroll
        for (int w = 1; w < 8; ++w) cs += colp[w * kTile + row];
        rs = seg_max(rs, seg);
        ra = seg_max(ra, seg);
        pm = seg_max(pm, seg);
        cs = seg_max(cs, seg);
        if (leader && half == 0) {
            atomicMax(&sh.stat[0][blk], ord_bits(rs));
            atomicMax(&sh.stat[1][blk], __float_as_uint(ra));
            atomicMax(&sh.stat[2][blk], __float_as_uint(cs));
            atomicMax(&sh.stat[3][blk], __float_as_uint(pm));
        }
    }
    __syncthreads();

    // V0 = c P (reference: c = 1.8 / (max_i sum_j P_ij)^2, :82-120, :176-178)
    // or c P^T (c = 1 / (||P||_1 ||P||_inf)).
    float sP = 1.f, sV = 1.f, pinf = 0.f, cinit = 0.f;
    if (valid) {
        const float rsmax = ord_float(sh.stat[0][blk]);
        const float ra = __uint_as_float(sh.stat[1][blk]);
        const float ca = __uint_as_float(sh.stat[2][blk]);
        const float pmax = __uint_as_float(sh.stat[3][blk]);
        cinit = (mode == LF_NS_INIT_REFERENCE) ? __fdiv_rn(1.8f, rsmax * rsmax) : __fdiv_rn(1.0f, ca * ra);
        sP = split_scale(pmax);
        sV = split_scale(fabsf(cinit) * pmax);  // max|V0| = |c| max|P|, exactly
        pinf = ra;
        if (leader && half == 0) atomicMax(&sh.vmax[0][blk], __float_as_uint(fabsf(cinit) * pmax));
    }
    const uint32_t tmem = sh.tmem_base;
    const uint32_t tl = (uint32_t)(quad * 32) << 16;  // this warp's TMEM lane quadrant
    float V[64];
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        float p[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 w = stage_ld4(stage, row, (c0 >> 2) + 4 * g + q);
            p[4 * q] = w.x; p[4 * q + 1] = w.y; p[4 * q + 2] = w.z; p[4 * q + 3] = w.w;
        }
        uint32_t pk[8];
        split_half(p, sP, false, pk);
        tmem_st8(tmem + tl + kTile + 32 * half + 8 * g, pk);
        split_half(p, sP, true, pk);
        tmem_st8(tmem + tl + kTile + 64 + 32 * half + 8 * g, pk);
#pragma unroll
        for (int j = 0; j < 16; ++j)
            V[16 * g + j] = cinit * ((mode == LF_NS_INIT_REFERENCE) ? p[j] : stage[stage_idx(c0 + 16 * g + j, row)]);
    }
    tmem_wait_st();
    bool ok = true;
    if (iters == 0) {
        if (valid) store_rows<T>(x + (m0 + blk) * (int64_t)n * n + (int64_t)(row - bn) * n, c0, bn, n, V);
    } else {
        tc_fence_before();
        __syncthreads();  // staging reads done (V's buffers overlap it); P in TMEM
        store_v(smem_u32(base) + rbase, rx, V, sV, precision == LF_NS_PREC_SPLIT3 || iters <= 2);
        fence_async_smem();
        tc_fence_before();
        __syncthreads();

        for (int k = 0; k < iters; ++k) {
            const uint32_t par = (uint32_t)k & 1u;
            const bool full = precision == LF_NS_PREC_SPLIT3 || k >= iters - 2;
            const bool last = k == iters - 1;
            // ---- H = P V -------------------------------------------------------
            if (warp == 0) {
                tc_fence_after();
                const uint32_t go = elect_one() ? 1u : 0u;
                const uint32_t sb = smem_u32(base);
                const uint64_t dvh = make_desc(sb, 16384, 1024), dvl = make_desc(sb + kOpBytes, 16384, 1024);
                if (full) issue_h<true>(tmem, tmem + kTile, tmem + kTile + 64, dvh, dvl, go);
                else issue_h<false>(tmem, tmem + kTile, tmem + kTile + 64, dvh, dvl, go);
                if (go) mma_commit(&sh.bar[0]);
                __syncwarp();
            }
            // the other parity's reduction slots were last read before the previous barrier
            if (tid < kTile) {
                sh.gmax[par ^ 1u][tid] = 0u;
                sh.vmax[par ^ 1u][tid] = 0u;
            }
            const float vmk = valid ? __uint_as_float(sh.vmax[par][blk]) : 0.f;
            const float sG = split_scale(1.f + pinf * vmk);  // |G_ij| <= 1 + ||P||_inf max|V|
            const float chs = -sG * (1.f / sP) * (1.f / sV);
            const uint64_t chs2 = pk2(chs, chs);
            bool okw = mbar_wait(&sh.bar[0], par);
            tc_fence_after();
            // ---- G = I - H (fp16, scaled) into shared memory --------------------
            __half2 hm = __float2half2_rn(0.f);
#pragma unroll
            for (int hp = 0; hp < 2; ++hp) {  // two 16-column loads per wait
                float av[16], aw[16];
                tmem_ld16(tmem + tl + c0 + 32 * hp, av);
                tmem_ld16(tmem + tl + c0 + 32 * hp + 16, aw);
                tmem_wait_ld();
                reg_fence(av);
                reg_fence(aw);
                const uint32_t gh_row = smem_u32(base) + 2 * kOpBytes + rbase;
                if (hp == dchunk) {
                    g_store<true>(av, chs2, sG, lane, 0, hm, gh_row, rx, 2 * hp);
                    g_store<true>(aw, chs2, sG, lane, 16, hm, gh_row, rx, 2 * hp + 1);
                } else {
                    g_store<false>(av, chs2, sG, lane, 0, hm, gh_row, rx, 2 * hp);
                    g_store<false>(aw, chs2, sG, lane, 0, hm, gh_row, rx, 2 * hp + 1);
                }
            }
            float gm = seg_max_nn(fmaxf(__low2float(hm), __high2float(hm)), seg, warp_one);
            if (leader) atomicMax(&sh.gmax[par][blk], __float_as_uint(gm));
            fence_async_smem();
            tc_fence_before();
            if (__syncthreads_or(!okw)) { ok = false; break; }
            // ---- Y = V G ---------------------------------------------------------
            if (warp == 0) {
                tc_fence_after();
                const uint32_t go = elect_one() ? 1u : 0u;
                const uint32_t sb = smem_u32(base);
                const uint64_t dvh = make_desc(sb, 16, 1024), dvl = make_desc(sb + kOpBytes, 16, 1024);
                const uint64_t dg = make_desc(sb + 2 * kOpBytes, 16384, 1024);
                if (full) issue_y<true>(tmem, dvh, dvl, dg, go);
                else issue_y<false>(tmem, dvh, dvl, dg, go);
                if (go) mma_commit(&sh.bar[1]);
                __syncwarp();
            }
            const float gmk = valid ? __uint_as_float(sh.gmax[par][blk]) * (1.f / sG) : 0.f;
            // max|V + V G| <= max|V| (1 + n max|G|); the 2^-11 rounding of the
            // fp16 maxima is far inside the factor-2 headroom of the scale
            const float sVn = split_scale(vmk * (1.f + (float)n * gmk));
            const uint64_t cy2 = pk2((1.f / sV) * (1.f / sG), (1.f / sV) * (1.f / sG));
            okw = mbar_wait(&sh.bar[1], par);
            tc_fence_after();
            // ---- V <- V + Y ------------------------------------------------------
#pragma unroll
            for (int hc = 0; hc < 4; ++hc) {
                float av[16];
                tmem_ld16(tmem + tl + c0 + 16 * hc, av);
                tmem_wait_ld();
                reg_fence(av);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const int j = 16 * hc + 2 * e;
                    upk2(fma2(pk2(av[2 * e], av[2 * e + 1]), cy2, pk2(V[j], V[j + 1])), V[j], V[j + 1]);
                }
            }
            if (last) {
                if (!okw) ok = false;
                else if (valid) store_rows<T>(x + (m0 + blk) * (int64_t)n * n + (int64_t)(row - bn) * n, c0, bn, n, V);
                break;
            }
            float vm = store_v(smem_u32(base) + rbase, rx, V, sVn, precision == LF_NS_PREC_SPLIT3 || k + 1 >= iters - 2) *
                       (1.f / sVn);
            vm = seg_max_nn(vm, seg, warp_one);
            if (leader) atomicMax(&sh.vmax[par ^ 1u][blk], __float_as_uint(vm));
            sV = sVn;
            fence_async_smem();
            tc_fence_before();
            if (__syncthreads_or(!okw)) { ok = false; break; }
        }
    }
    if (!ok) atomicExch(&g_ns_status, (int)LF_ERR_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ---------------------------------------------------------------------------
// CUDA-core kernels
// ---------------------------------------------------------------------------
constexpr int kRB = 16;  // rows per block in the row-blocked products

// Block-wide reductions used in set-up.
template <typename Acc>
__device__ Acc block_reduce_max(Acc v, Acc* red) {
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    Acc m = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) m = max(m, red[w]);
    return m;
}

// V resident in shared memory as Acc [n][n+1]; the new iterate goes to a
// second shared buffer, or to the output (type T == Acc) when two buffers do
// not fit.  W = V P (P read from A on the fly) and Y = W V are formed 16 rows
// at a time: the reference's (V P) V association.
template <typename T, typename Acc, bool NEWV_GLOBAL>
__global__ void __launch_bounds__(256)
ns_simt_fwd_kernel(const T* __restrict__ a, T* __restrict__ x, int n, int iters, int mode, Acc reg) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int S = n + 1;
    Acc* V = reinterpret_cast<Acc*>(smem_raw);
    Acc* Vn = V + (size_t)n * S;                      // only when !NEWV_GLOBAL
    Acc* Wr = Vn + (NEWV_GLOBAL ? 0 : (size_t)n * S); // kRB x S
    Acc* red = Wr + kRB * S;                          // 8 entries
    const int tid = threadIdx.x;
    const int64_t mat = blockIdx.x;
    const T* A = a + mat * (int64_t)n * n;
    T* X = x + mat * (int64_t)n * n;
    auto P = [&](int i, int j) -> Acc { return (Acc)Elem<T>::load(A[(int64_t)i * n + j]) + (i == j ? reg : Acc(0)); };

    // Initialisation.
    Acc c0;
    if (mode == LF_NS_INIT_REFERENCE) {
        Acc mx = Acc(-1e30);
        for (int i = tid; i < n; i += blockDim.x) {
            Acc s = 0;
            for (int j = 0; j < n; ++j) s += P(i, j);
            mx = max(mx, s);
        }
        mx = block_reduce_max<Acc>(mx, red);
        c0 = Acc(1.8) / (mx * mx);
    } else {
        Acc r1 = 0, ri = 0;
        for (int i = tid; i < n; i += blockDim.x) {
            Acc rs = 0, cs = 0;
            for (int j = 0; j < n; ++j) { rs += fabs(P(i, j)); cs += fabs(P(j, i)); }
            ri = max(ri, rs);
            r1 = max(r1, cs);
        }
        ri = block_reduce_max<Acc>(ri, red);
        r1 = block_reduce_max<Acc>(r1, red);
        c0 = Acc(1) / (r1 * ri);
    }
    for (int e = tid; e < n * n; e += blockDim.x) {
        int i = e / n, j = e - i * n;
        V[i * S + j] = (mode == LF_NS_INIT_REFERENCE ? P(i, j) : P(j, i)) * c0;
    }
    __syncthreads();

    const int tpr = blockDim.x / kRB;  // threads per row of the block (16)
    const int rr = tid / tpr, tj = tid - rr * tpr;
    for (int it = 0; it < iters; ++it) {
        for (int r0 = 0; r0 < n; r0 += kRB) {
            const int r = r0 + rr;
            // W[rr][j] = sum_k V[r][k] P[k][j]
            for (int j = tj; j < n; j += tpr) {
                Acc acc = 0;
                if (r < n)
                    for (int k = 0; k < n; ++k) acc = fma_acc(V[r * S + k], P(k, j), acc);
                Wr[rr * S + j] = acc;
            }
            __syncthreads();
            // Y[r][j] = sum_k W[rr][k] V[k][j];  V'[r][j] = 2 V[r][j] - Y
            if (r < n) {
                for (int j = tj; j < n; j += tpr) {
                    Acc acc = 0;
                    for (int k = 0; k < n; ++k) acc = fma_acc(Wr[rr * S + k], V[k * S + j], acc);
                    Acc vn = fma_acc(Acc(2), V[r * S + j], -acc);
                    if (NEWV_GLOBAL) X[(int64_t)r * n + j] = (T)vn;
                    else Vn[r * S + j] = vn;
                }
            }
            __syncthreads();
        }
        if (NEWV_GLOBAL) {
            __threadfence_block();
            for (int e = tid; e < n * n; e += blockDim.x) {
                int i = e / n, j = e - i * n;
                V[i * S + j] = (Acc)X[e];
            }
        } else {
            for (int e = tid; e < n * n; e += blockDim.x) {
                int i = e / n, j = e - i * n;
                V[i * S + j] = Vn[i * S + j];
            }
        }
        __syncthreads();
    }
    for (int e = tid; e < n * n; e += blockDim.x) {
        int i = e / n, j = e - i * n;
        X[e] = Elem<T>::store(V[i * S + j]);
    }
}

// dA = -(V^T G) V^T, V resident in shared memory, G read from global.
template <typename T, typename Acc>
__global__ void __launch_bounds__(256)
ns_simt_bwd_kernel(const T* __restrict__ g, const T* __restrict__ v, T* __restrict__ da, int n) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int S = n + 1;
    Acc* V = reinterpret_cast<Acc*>(smem_raw);
    Acc* Tr = V + (size_t)n * S;
    const int tid = threadIdx.x;
    const int64_t mat = blockIdx.x;
    const T* G = g + mat * (int64_t)n * n;
    const T* Vg = v + mat * (int64_t)n * n;
    T* O = da + mat * (int64_t)n * n;
    for (int e = tid; e < n * n; e += blockDim.x) {
        int i = e / n, j = e - i * n;
        V[i * S + j] = (Acc)Elem<T>::load(Vg[e]);
    }
    __syncthreads();
    const int tpr = blockDim.x / kRB;
    const int rr = tid / tpr, tj = tid - rr * tpr;
    for (int r0 = 0; r0 < n; r0 += kRB) {
        const int r = r0 + rr;
        for (int j = tj; j < n; j += tpr) {
            Acc acc = 0;
            if (r < n)
                for (int p = 0; p < n; ++p) acc = fma_acc(V[p * S + r], (Acc)Elem<T>::load(G[(int64_t)p * n + j]), acc);
            Tr[rr * S + j] = acc;
        }
        __syncthreads();
        if (r < n) {
            for (int j = tj; j < n; j += tpr) {
                Acc acc = 0;
                for (int k = 0; k < n; ++k) acc = fma_acc(Tr[rr * S + k], V[j * S + k], acc);
                O[(int64_t)r * n + j] = Elem<T>::store(-acc);
            }
        }
        __syncthreads();
    }
}

// res[b] = ||(A + reg I) X - I||_F, accumulated in Acc.
template <typename T, typename Acc>
__global__ void __launch_bounds__(256)
ns_residual_kernel(const T* __restrict__ a, const T* __restrict__ x, Acc* __restrict__ res, int n, Acc reg) {
    __shared__ Acc red[8];
    const int64_t mat = blockIdx.x;
    const T* A = a + mat * (int64_t)n * n;
    const T* X = x + mat * (int64_t)n * n;
    Acc ss = 0;
    for (int e = threadIdx.x; e < n * n; e += blockDim.x) {
        int i = e / n, j = e - i * n;
        Acc acc = 0;
        for (int k = 0; k < n; ++k)
            acc = fma_acc((Acc)Elem<T>::load(A[(int64_t)i * n + k]) + (i == k ? reg : Acc(0)),
                      (Acc)Elem<T>::load(X[(int64_t)k * n + j]), acc);
        acc -= (i == j) ? Acc(1) : Acc(0);
        ss = fma_acc(acc, acc, ss);
    }
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        Acc t = 0;
        for (int w = 0; w < 8; ++w) t += red[w];
        res[mat] = sqrt(t);
    }
}

// ---------------------------------------------------------------------------
// Backward on tcgen05: dA = -(V^T G) V^T (reference :469-573), n <= 128.
// One CTA per 128x128 tile (floor(128/n) matrices on the diagonal for
// n <= 64).  V and G are split as hi + lo fp16 with per-matrix scales and
// stored row-major with the 128-byte swizzle; the transposes come from the
// descriptor views of the same bytes:
//   T1 = V^T G   A = V as an MN-major operand (A[m][k] = V[k][m]), B = G MN-major
//   dA = -T1 V^T A = T1 from tensor memory (hi/lo fp16), B = V as a K-major
//                operand (B[k][n] = V[n][k])
// each as hi*hi + hi*lo + lo*hi (the split3 arithmetic of the forward).
// ---------------------------------------------------------------------------
constexpr uint32_t kIdescT1 = (1u << 4) | (1u << 15) | (1u << 16) | ((uint32_t)(kTile >> 3) << 17) |
                              ((uint32_t)(kTile >> 4) << 24);  // A and B MN-major
constexpr uint32_t kIdescDA = (1u << 4) | ((uint32_t)(kTile >> 3) << 17) | ((uint32_t)(kTile >> 4) << 24);  // B K-major

struct NsBwdShared {
    uint64_t bar[2];
    uint32_t tmem_base;
    uint32_t vmax[kTile], gmax[kTile], tmax[kTile];  // per matrix of the tile (float bits)
};

// Row `row`, 64 columns of the matrix at src (rows of the tile's matrices,
// zero outside the row's own matrix) into v.
template <typename T>
__device__ __forceinline__ void load_rows(const T* __restrict__ src, int64_t m0, int n, bool valid, int blk, int bn,
                                          int row, int c0, float (&v)[64]) {
#pragma unroll
    for (int j = 0; j < 64; ++j) v[j] = 0.f;
    if (!valid) return;
    const T* r = src + ((m0 + blk) * (int64_t)n + (row - bn)) * n - bn;  // r[c], c in [bn, bn+n)
    if constexpr (sizeof(T) == 4) {
        if (n == kTile && (reinterpret_cast<uintptr_t>(r + c0) & 15) == 0) {
#pragma unroll
            for (int j = 0; j < 64; j += 4) {
                const float4 w = *reinterpret_cast<const float4*>(r + c0 + j);
                v[j] = w.x; v[j + 1] = w.y; v[j + 2] = w.z; v[j + 3] = w.w;
            }
            return;
        }
    }
#pragma unroll
    for (int j = 0; j < 64; ++j)
        if ((unsigned)(c0 + j - bn) < (unsigned)n) v[j] = Elem<T>::load(r[c0 + j]);
}

__device__ __forceinline__ float abs_max64(const float (&v)[64]) {
    float m0 = 0.f, m1 = 0.f;
#pragma unroll
    for (int j = 0; j < 64; j += 2) {
        m0 = fmaxf(m0, fabsf(v[j]));
        m1 = fmaxf(m1, fabsf(v[j + 1]));
    }
    return fmaxf(m0, m1);
}

template <typename T>
__global__ void __launch_bounds__(kTcThreads, 1)
ns_tc_bwd_kernel(const T* __restrict__ g, const T* __restrict__ v, T* __restrict__ da, int batch, int n, int nb) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    NsBwdShared& sh = *reinterpret_cast<NsBwdShared*>(base + 4 * kOpBytes);
    const uint32_t sb = smem_u32(base);  // V hi, V lo, G hi, G lo: 32 KB each

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quad = warp & 3, half = warp >> 2;
    const int row = quad * 32 + lane;
    const int c0 = half * 64;
    const uint32_t rbase = (uint32_t)(half * 16384 + row * 128);
    const int rx = row & 7;
    const int64_t m0 = (int64_t)blockIdx.x * nb;
    const int nrows = (int)min((int64_t)nb, (int64_t)batch - m0) * n;
    const bool valid = row < nrows;
    const int blk = valid ? row / n : -1;
    const int bn = valid ? blk * n : 0;

    if (tid == 0) {
        mbar_init(&sh.bar[0], 1);
        mbar_init(&sh.bar[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int e = tid; e < kTile; e += kTcThreads) sh.vmax[e] = sh.gmax[e] = sh.tmax[e] = 0u;
    if (warp == 0) tmem_alloc(&sh.tmem_base, kTmemCols);
    uint32_t seg = 0;
#pragma unroll
    for (int i = 0; i < 5; ++i) {
        const int o = __shfl_down_sync(0xffffffffu, blk, 1 << i);
        if (valid && lane + (1 << i) < 32 && o == blk) seg |= 1u << i;
    }
    const int prev = __shfl_up_sync(0xffffffffu, blk, 1);
    const bool leader = valid && (lane == 0 || prev != blk);
    const int blk0 = __shfl_sync(0xffffffffu, blk, 0);
    const bool warp_one = __all_sync(0xffffffffu, valid && blk == blk0);

    // ---- V and G rows, their per-matrix maxima ------------------------------
    float w[64];
    load_rows<T>(v, m0, n, valid, blk, bn, row, c0, w);
    {
        const float m = seg_max_nn(abs_max64(w), seg, warp_one);
        if (leader) atomicMax(&sh.vmax[blk], __float_as_uint(m));
    }
    __syncthreads();
    const float sV = valid ? split_scale(__uint_as_float(sh.vmax[blk])) : 1.f;
    store_v(sb + rbase, rx, w, sV, true);  // V hi at [0,32K), lo at [32K,64K)
    load_rows<T>(g, m0, n, valid, blk, bn, row, c0, w);
    {
        const float m = seg_max_nn(abs_max64(w), seg, warp_one);
        if (leader) atomicMax(&sh.gmax[blk], __float_as_uint(m));
    }
    __syncthreads();
    const float sG = valid ? split_scale(__uint_as_float(sh.gmax[blk])) : 1.f;
    store_v(sb + 2 * kOpBytes + rbase, rx, w, sG, true);  // G hi at [64K,96K), lo at [96K,128K)
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    const uint32_t tmem = sh.tmem_base;
    const uint32_t tl = (uint32_t)(quad * 32) << 16;
    bool ok = true;

    // ---- T1 = V^T G --------------------------------------------------------
    if (warp == 0) {
        tc_fence_after();
        const uint32_t go = elect_one() ? 1u : 0u;
        const uint64_t dvh = make_desc(sb, 16384, 1024), dvl = make_desc(sb + kOpBytes, 16384, 1024);
        const uint64_t dgh = make_desc(sb + 2 * kOpBytes, 16384, 1024), dgl = make_desc(sb + 3 * kOpBytes, 16384, 1024);
#pragma unroll
        for (int ks = 0; ks < kTile / 16; ++ks) {
            const uint64_t o = (uint64_t)(ks * 128);  // K step = 16 rows of both row-major operands
            mma_f16(tmem, dvh + o, dgh + o, kIdescT1, ks > 0 ? 1u : 0u, go);
            mma_f16(tmem, dvh + o, dgl + o, kIdescT1, 1u, go);
            mma_f16(tmem, dvl + o, dgh + o, kIdescT1, 1u, go);
        }
        if (go) mma_commit(&sh.bar[0]);
        __syncwarp();
    }
    ok = mbar_wait(&sh.bar[0], 0);
    ok = !__syncthreads_or(!ok);
    tc_fence_after();
    // T1 = acc / (sV sG); its hi/lo parts go to tensor memory as the next A operand
    float t[64];
#pragma unroll
    for (int hc = 0; hc < 4; ++hc) {
        float av[16];
        tmem_ld16(tmem + tl + c0 + 16 * hc, av);
        tmem_wait_ld();
        reg_fence(av);
#pragma unroll
        for (int j = 0; j < 16; ++j) t[16 * hc + j] = av[j];
    }
    {
        const float m = seg_max_nn(abs_max64(t), seg, warp_one);
        if (leader) atomicMax(&sh.tmax[blk], __float_as_uint(m));
    }
    __syncthreads();
    const float sT = valid ? split_scale(__uint_as_float(sh.tmax[blk])) : 1.f;  // of the accumulator values
#pragma unroll
    for (int hc = 0; hc < 4; ++hc) {
        float p[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) p[j] = t[16 * hc + j];
        uint32_t pk[8];
        split_half(p, sT, false, pk);
        tmem_st8(tmem + tl + kTile + 32 * half + 8 * hc, pk);
        split_half(p, sT, true, pk);
        tmem_st8(tmem + tl + kTile + 64 + 32 * half + 8 * hc, pk);
        tmem_wait_st();
    }
    tc_fence_before();
    __syncthreads();
    // ---- dA = -T1 V^T ------------------------------------------------------
    if (warp == 0) {
        tc_fence_after();
        const uint32_t el = elect_one() ? 1u : 0u;  // every lane of the warp elects
        const uint32_t go = ok ? el : 0u;
        const uint64_t dvh = make_desc(sb, 16, 1024), dvl = make_desc(sb + kOpBytes, 16, 1024);
#pragma unroll
        for (int ks = 0; ks < kTile / 16; ++ks) {
            const uint64_t bo = (uint64_t)((ks >> 2) * 1024 + (ks & 3) * 2);  // K-major: 32 bytes per K step
            mma_f16_ts(tmem, tmem + kTile + ks * 8, dvh + bo, kIdescDA, ks > 0 ? 1u : 0u, go);
            mma_f16_ts(tmem, tmem + kTile + ks * 8, dvl + bo, kIdescDA, 1u, go);
            mma_f16_ts(tmem, tmem + kTile + 64 + ks * 8, dvh + bo, kIdescDA, 1u, go);
        }
        if (go) mma_commit(&sh.bar[1]);
        __syncwarp();
    }
    if (ok) ok = mbar_wait(&sh.bar[1], 0);
    ok = !__syncthreads_or(!ok);
    tc_fence_after();
    // acc = T1 V^T * (sV sG) sT sV  ->  dA = -acc / (sV sG sT sV)
    const float cd = -(1.f / sV) * (1.f / sG) * (1.f / sT) * (1.f / sV);
#pragma unroll
    for (int hc = 0; hc < 4; ++hc) {
        float av[16];
        tmem_ld16(tmem + tl + c0 + 16 * hc, av);
        tmem_wait_ld();
        reg_fence(av);
#pragma unroll
        for (int j = 0; j < 16; ++j) t[16 * hc + j] = av[j] * cd;
    }
    if (ok && valid) store_rows<T>(da + ((m0 + blk) * (int64_t)n + (row - bn)) * n, c0, bn, n, t);
    if (!ok && tid == 0) atomicExch(&g_ns_status, (int)LF_ERR_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

size_t tc_bwd_smem_bytes() { return 4 * (size_t)kOpBytes + sizeof(NsBwdShared) + 1024; }

template <typename T>
int launch_tc_bwd(const void* g, const void* v, void* da, int64_t batch, int64_t n, cudaStream_t st) {
    const size_t smem = tc_bwd_smem_bytes();
    if (smem > (size_t)max_optin_smem()) {
        set_error("NewtonInverse backward tensor-core path needs %zu bytes of shared memory", smem);
        return LF_ERR_UNSUPPORTED;
    }
    const int nb = tc_per_tile(n);
    const int64_t tiles = (batch + nb - 1) / nb;
    auto kern = ns_tc_bwd_kernel<T>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kern<<<(unsigned)tiles, kTcThreads, smem, st>>>(static_cast<const T*>(g), static_cast<const T*>(v),
                                                   static_cast<T*>(da), (int)batch, (int)n, nb);
    return check_launch("ns_tc_bwd_kernel");
}

// ---------------------------------------------------------------------------
// Matrices with 128 < n <= 256 (fp32) on tcgen05: a cluster of four CTAs per
// matrix.  The matrix is zero padded to 256 = 2 x 2 blocks of 128; CTA
// (I, J) (cluster rank 2I + J) owns block (I, J) of H, G, Y and V:
//   H_IJ = P_I0 V_0J + P_I1 V_1J      A = P rows I (all 256 columns) in tensor memory
//   G_IJ = delta_IJ - H_IJ
//   Y_IJ = V_I0 G_0J + V_I1 G_1J      A = V tiles, B = G tiles, shared memory
//   V_IJ += Y_IJ
// Each product needs one tile a peer owns: V_(1-I)J for H, V_I(1-J) and
// G_(1-I)J for Y.  They are pulled over distributed shared memory (mapa +
// ld.shared::cluster) into local buffers, so no global scratch is needed
// (the C ABI allocates nothing).  Scales and maxima are per matrix: each CTA
// reduces its block, the four blocks meet through distributed shared memory
// after the cluster barriers that already separate the phases.  Every CTA
// executes every cluster barrier whatever happens to its own waits (a timed
// out wait only skips MMA work), so no CTA can leave a peer waiting.
// ---------------------------------------------------------------------------
constexpr int kC256Threads = 256;
constexpr int kC256TmemCols = 512;  // accumulator [0,128), P hi [128,256), P lo [256,384)
// shared memory (from the 1024-aligned base): own V hi/lo [0,64K), peer V
// hi/lo [64K,128K), own G hi [128K,160K), peer G hi [160K,192K)
constexpr uint32_t kOwnV = 0, kExtV = 2 * kOpBytes, kOwnG = 4 * kOpBytes, kExtG = 5 * kOpBytes;

struct Ns256Shared {
    uint64_t bar[2];           // [0]: H complete, [1]: Y complete
    uint32_t tmem_base;
    uint32_t gmax[2];          // this CTA's block max|G * sG| (float bits), by iteration parity
    uint32_t vmax[2];          // this CTA's block max|V| (float bits), by iteration parity
    uint32_t stat[4];          // set-up, this CTA's rows: max signed row sum (ordered), max |row| sum, max|P|, unused
    float colpart[2 * kTile];  // set-up: this CTA's |column| sums over its 128 rows, all 256 columns
};

__device__ __forceinline__ uint32_t cluster_addr(uint32_t local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}
__device__ __forceinline__ uint32_t ld_cluster_u32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
    return v;
}
__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) { return __uint_as_float(ld_cluster_u32(addr)); }
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Copies `bytes` (a multiple of 16 KB) at shared offset `src` of cluster CTA
// `rank` to local shared offset `dst`; all threads of the CTA take part.
__device__ __forceinline__ void pull_tile(uint32_t sb, uint32_t dst, uint32_t src, uint32_t rank, int bytes) {
    const uint32_t rsrc = cluster_addr(sb + src, rank);
    for (int base = threadIdx.x * 16; base < bytes; base += kC256Threads * 16 * 4) {
        uint32_t v[4][4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
            asm volatile("ld.shared::cluster.v4.u32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(v[u][0]), "=r"(v[u][1]), "=r"(v[u][2]), "=r"(v[u][3])
                         : "r"(rsrc + base + u * kC256Threads * 16)
                         : "memory");
#pragma unroll
        for (int u = 0; u < 4; ++u) sts128(sb + dst + base + u * kC256Threads * 16, v[u][0], v[u][1], v[u][2], v[u][3]);
    }
}

// H (+)= sum over the two K blocks of P_I,kb (tensor memory: hi columns
// a_hi + 64 kb + 8 ks) times V_kb,J (descriptors dvh[kb], dvl[kb]).
template <bool FULL>
__device__ __forceinline__ void issue_h256(uint32_t acc, uint32_t a_hi, uint32_t a_lo, const uint64_t (&dvh)[2],
                                           const uint64_t (&dvl)[2], uint32_t go) {
#pragma unroll
    for (int kb = 0; kb < 2; ++kb)
#pragma unroll
        for (int ks = 0; ks < kTile / 16; ++ks) {
            const uint32_t ac = 64 * kb + 8 * ks;
            const uint64_t bo = (uint64_t)(ks * 128);
            mma_f16_ts(acc, a_hi + ac, dvh[kb] + bo, kIdesc, (kb | ks) ? 1u : 0u, go);
            if (FULL) {
                mma_f16_ts(acc, a_hi + ac, dvl[kb] + bo, kIdesc, 1u, go);
                mma_f16_ts(acc, a_lo + ac, dvh[kb] + bo, kIdesc, 1u, go);
            }
        }
}

// Y (+)= sum over the two K blocks of V_I,kb (K-major, dah[kb] / dal[kb])
// times G_kb,J (MN-major, dg[kb]).
template <bool FULL>
__device__ __forceinline__ void issue_y256(uint32_t acc, const uint64_t (&dah)[2], const uint64_t (&dal)[2],
                                           const uint64_t (&dg)[2], uint32_t go) {
#pragma unroll
    for (int kb = 0; kb < 2; ++kb)
#pragma unroll
        for (int ks = 0; ks < kTile / 16; ++ks) {
            const uint64_t ao = (uint64_t)((ks >> 2) * 1024 + (ks & 3) * 2);
            mma_f16(acc, dah[kb] + ao, dg[kb] + (uint64_t)(ks * 128), kIdesc, (kb | ks) ? 1u : 0u, go);
            if (FULL) mma_f16(acc, dal[kb] + ao, dg[kb] + (uint64_t)(ks * 128), kIdesc, 1u, go);
        }
}

__global__ void __cluster_dims__(4, 1, 1) __launch_bounds__(kC256Threads, 1)
ns_tc256_fwd_kernel(const float* __restrict__ a, float* __restrict__ x, int n, int iters, int mode, float reg,
                    int precision) {
    extern __shared__ __align__(16) unsigned char smem_raw[];  // re-aligned to 1024 below
    unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* stage = reinterpret_cast<float*>(base + kExtV);  // set-up: rows I of P, 128 x 256 fp32 (128 KB)
    Ns256Shared& sh = *reinterpret_cast<Ns256Shared*>(base + 6 * kOpBytes);
    const uint32_t sb = smem_u32(base);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quad = warp & 3, half = warp >> 2;
    const int row = quad * 32 + lane;  // row of the block (= TMEM lane)
    const int c0 = half * 64;          // this thread's 64 columns of the block
    const uint32_t rbase = (uint32_t)(half * 16384 + row * 128);
    const int rx = row & 7;
    const uint32_t crank = blockIdx.x & 3u;  // cluster rank = 2 I + J
    const int I = (int)(crank >> 1), J = (int)(crank & 1);
    const int64_t mat = blockIdx.x >> 2;
    const float* A = a + mat * (int64_t)n * n;
    float* X = x + mat * (int64_t)n * n;
    const int gi = 128 * I + row;  // matrix row of this thread
    const bool rvalid = gi < n;
    const int dchunk = (I == J && (quad >> 1) == half) ? (quad & 1) : -1;  // diagonal chunk (diagonal blocks only)
    const uint32_t rank_vi = (uint32_t)(2 * (1 - I) + J);  // owner of V_(1-I)J and G_(1-I)J
    const uint32_t rank_vj = (uint32_t)(2 * I + (1 - J));  // owner of V_I(1-J)

    if (tid == 0) {
        mbar_init(&sh.bar[0], 1);
        mbar_init(&sh.bar[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        sh.gmax[0] = sh.gmax[1] = sh.vmax[0] = sh.vmax[1] = 0u;
        sh.stat[0] = sh.stat[1] = sh.stat[2] = sh.stat[3] = 0u;
    }
    if (warp == 0) tmem_alloc(&sh.tmem_base, kC256TmemCols);

    // ---- set-up: rows I of P = A + reg I (all 256 columns) into the stage ----
    // stage row r, column c (0..255) at r*256 + swizzled chunk (16-byte chunks XOR r%32 within each 128-column half)
    auto st_idx = [](int r, int c) { return r * 256 + (c & 128) + ((((c & 127) >> 2) ^ r) & 31) * 4 + (c & 3); };
    for (int e = tid; e < kTile * 64; e += kC256Threads) {  // 64 float4 per row
        const int r = e >> 6, c4 = e & 63, c = 4 * c4;
        const int i = 128 * I + r;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < n) {
            const float* Ar = A + (int64_t)i * n;
            float* vp = &v.x;
            if ((n & 3) == 0 && c + 3 < n) {
                v = *reinterpret_cast<const float4*>(Ar + c);
            } else {
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    if (c + q < n) vp[q] = Ar[c + q];
            }
            if (i >= c && i < c + 4) vp[i - c] += reg;
        }
        *reinterpret_cast<float4*>(stage + st_idx(r, c)) = v;
    }
    __syncthreads();
    // this CTA's rows: signed row sum, |row| sum, max|P|; |column| partial sums
    {
        if (tid < kTile) {
            float rs = 0.f, ra = 0.f, pm = 0.f;
            for (int c = 0; c < 2 * kTile; ++c) {
                const float p = stage[st_idx(tid, c)];
                rs += p;
                ra += fabsf(p);
                pm = fmaxf(pm, fabsf(p));
            }
            if (128 * I + tid < n) {
                atomicMax(&sh.stat[0], ord_bits(rs));
                atomicMax(&sh.stat[1], __float_as_uint(ra));
            }
            atomicMax(&sh.stat[2], __float_as_uint(pm));
        }
        for (int c = tid; c < 2 * kTile; c += kC256Threads) {
            float cs = 0.f;
            for (int r = 0; r < kTile; ++r) cs += fabsf(stage[st_idx(r, c)]);
            sh.colpart[c] = cs;
        }
    }
    cluster_sync_all();  // every CTA's statistics are visible to its peers
    float rsmax = -INFINITY, ramax = 0.f, pmax = 0.f, camax = 0.f;
    {
        const uint32_t sst = smem_u32(&sh.stat[0]), scol = smem_u32(&sh.colpart[0]);
#pragma unroll
        for (uint32_t rk = 0; rk < 4; ++rk) {
            rsmax = fmaxf(rsmax, ord_float(ld_cluster_u32(cluster_addr(sst, rk))));
            ramax = fmaxf(ramax, ld_cluster_f32(cluster_addr(sst + 4, rk)));
            pmax = fmaxf(pmax, ld_cluster_f32(cluster_addr(sst + 8, rk)));
        }
        // full |column| sums = this row half + the other row half (ranks 0/2 hold rows 0..127 / 128..255)
        for (int c = lane; c < 2 * kTile; c += 32) {
            const float cs = ld_cluster_f32(cluster_addr(scol + 4 * c, 0)) + ld_cluster_f32(cluster_addr(scol + 4 * c, 2));
            camax = fmaxf(camax, cs);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) camax = fmaxf(camax, __shfl_xor_sync(0xffffffffu, camax, o));
    }
    const float cinit = (mode == LF_NS_INIT_REFERENCE) ? __fdiv_rn(1.8f, rsmax * rsmax) : __fdiv_rn(1.0f, camax * ramax);
    const float sP = split_scale(pmax);
    float sV = split_scale(fabsf(cinit) * pmax);
    const float pinf = ramax;
    float vmk = fabsf(cinit) * pmax;  // max|V0|
    const uint32_t tmem = sh.tmem_base;
    const uint32_t tl = (uint32_t)(quad * 32) << 16;
    // P rows I as the A operand: K columns kb*128 + c0 + [0,64) of each K block
#pragma unroll
    for (int kb = 0; kb < 2; ++kb)
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            float p[16];
#pragma unroll
            for (int q = 0; q < 16; ++q) p[q] = stage[st_idx(row, 128 * kb + c0 + 16 * g + q)];
            uint32_t pk[8];
            split_half(p, sP, false, pk);
            tmem_st8(tmem + tl + kTile + 64 * kb + 32 * half + 8 * g, pk);
            split_half(p, sP, true, pk);
            tmem_st8(tmem + tl + 2 * kTile + 64 * kb + 32 * half + 8 * g, pk);
            tmem_wait_st();
        }
    // V0 block (I, J): c P_IJ, or c (P_JI)^T read from the input
    float V[64];
#pragma unroll
    for (int j = 0; j < 64; ++j) {
        const int gc = 128 * J + c0 + j;
        float pv;
        if (mode == LF_NS_INIT_REFERENCE) {
            pv = stage[st_idx(row, 128 * J + c0 + j)];
        } else {
            pv = (rvalid && gc < n) ? A[(int64_t)gc * n + gi] + (gc == gi ? reg : 0.f) : 0.f;
        }
        V[j] = cinit * pv;
    }
    bool ok = true;
    if (iters == 0) {
        if (rvalid)
            for (int j = 0; j < 64; ++j)
                if (128 * J + c0 + j < n) X[(int64_t)gi * n + 128 * J + c0 + j] = V[j];
    } else {
        tc_fence_before();
        __syncthreads();  // stage reads done: the stage overlaps the peer buffers
        store_v(sb + kOwnV + rbase, rx, V, sV, precision == LF_NS_PREC_SPLIT3 || iters <= 2);
        fence_async_smem();
        for (int k = 0; k < iters; ++k) {
            const uint32_t par = (uint32_t)k & 1u;
            const bool full = precision == LF_NS_PREC_SPLIT3 || k >= iters - 2;
            const bool last = k == iters - 1;
            const int vbytes = full ? 2 * kOpBytes : kOpBytes;
            // ---- pull V_(1-I)J; H = P V -------------------------------------
            cluster_sync_all();  // X1: every block's V_k (and its max) is complete
            if (k > 0) {
                vmk = 0.f;
#pragma unroll
                for (uint32_t rk = 0; rk < 4; ++rk)
                    vmk = fmaxf(vmk, ld_cluster_f32(cluster_addr(smem_u32(&sh.vmax[par]), rk)));
            }
            if (tid == 0) sh.gmax[par] = 0u;  // last read by the peers before X1
            pull_tile(sb, kExtV, kOwnV, rank_vi, vbytes);
            fence_async_smem();
            tc_fence_before();
            __syncthreads();
            if (warp == 0) {
                tc_fence_after();
                const uint32_t el = elect_one() ? 1u : 0u;  // every lane of the warp elects
                const uint32_t go = ok ? el : 0u;
                uint64_t dvh[2], dvl[2];
                dvh[I] = make_desc(sb + kOwnV, 16384, 1024);
                dvl[I] = make_desc(sb + kOwnV + kOpBytes, 16384, 1024);
                dvh[1 - I] = make_desc(sb + kExtV, 16384, 1024);
                dvl[1 - I] = make_desc(sb + kExtV + kOpBytes, 16384, 1024);
                if (full) issue_h256<true>(tmem, tmem + kTile, tmem + 2 * kTile, dvh, dvl, go);
                else issue_h256<false>(tmem, tmem + kTile, tmem + 2 * kTile, dvh, dvl, go);
                if (go) mma_commit(&sh.bar[0]);
                __syncwarp();
            }
            const float sG = split_scale(1.f + pinf * vmk);  // |G_ij| <= 1 + ||P||_inf max|V|
            const float chs = -sG * (1.f / sP) * (1.f / sV);
            const uint64_t chs2 = pk2(chs, chs);
            if (ok) ok = mbar_wait(&sh.bar[0], par);
            ok = !__syncthreads_or(!ok);
            tc_fence_after();
            // ---- G_IJ into the own G buffer --------------------------------
            __half2 hm = __float2half2_rn(0.f);
#pragma unroll
            for (int hc = 0; hc < 4; ++hc) {
                float av[16];
                tmem_ld16(tmem + tl + c0 + 16 * hc, av);
                tmem_wait_ld();
                reg_fence(av);
                const uint32_t gh_row = sb + kOwnG + rbase;
                if ((hc >> 1) == dchunk) g_store<true>(av, chs2, sG, lane, 16 * (hc & 1), hm, gh_row, rx, hc);
                else g_store<false>(av, chs2, sG, lane, 0, hm, gh_row, rx, hc);
            }
            {
                const float gm = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(fmaxf(__low2float(hm), __high2float(hm)))));
                if (lane == 0) atomicMax(&sh.gmax[par], __float_as_uint(gm));
            }
            tc_fence_before();
            __syncthreads();  // H consumed; the peer V buffer is free again
            pull_tile(sb, kExtV, kOwnV, rank_vj, vbytes);  // V_I(1-J)
            fence_async_smem();
            // ---- pull G_(1-I)J; Y = V G ----------------------------------------
            cluster_sync_all();  // X2: every G block and its max are complete; the V pulls are done
            if (tid == 0) sh.vmax[par ^ 1u] = 0u;  // last read by the peers after the previous X1
            pull_tile(sb, kExtG, kOwnG, rank_vi, kOpBytes);
            float gmk = 0.f;
#pragma unroll
            for (uint32_t rk = 0; rk < 4; ++rk) gmk = fmaxf(gmk, ld_cluster_f32(cluster_addr(smem_u32(&sh.gmax[par]), rk)));
            gmk *= 1.f / sG;
            fence_async_smem();
            tc_fence_before();
            __syncthreads();
            if (warp == 0) {
                tc_fence_after();
                const uint32_t el = elect_one() ? 1u : 0u;
                const uint32_t go = ok ? el : 0u;
                uint64_t dah[2], dal[2], dg[2];
                dah[J] = make_desc(sb + kOwnV, 16, 1024);
                dal[J] = make_desc(sb + kOwnV + kOpBytes, 16, 1024);
                dah[1 - J] = make_desc(sb + kExtV, 16, 1024);
                dal[1 - J] = make_desc(sb + kExtV + kOpBytes, 16, 1024);
                dg[I] = make_desc(sb + kOwnG, 16384, 1024);
                dg[1 - I] = make_desc(sb + kExtG, 16384, 1024);
                if (full) issue_y256<true>(tmem, dah, dal, dg, go);
                else issue_y256<false>(tmem, dah, dal, dg, go);
                if (go) mma_commit(&sh.bar[1]);
                __syncwarp();
            }
            const float sVn = split_scale(vmk * (1.f + (float)n * gmk));  // max|V + V G| <= max|V| (1 + n max|G|)
            const uint64_t cy2 = pk2((1.f / sV) * (1.f / sG), (1.f / sV) * (1.f / sG));
            if (ok) ok = mbar_wait(&sh.bar[1], par);
            ok = !__syncthreads_or(!ok);
            tc_fence_after();
            // ---- V_IJ += Y_IJ ------------------------------------------------
#pragma unroll
            for (int hc = 0; hc < 4; ++hc) {
                float av[16];
                tmem_ld16(tmem + tl + c0 + 16 * hc, av);
                tmem_wait_ld();
                reg_fence(av);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const int j = 16 * hc + 2 * e;
                    upk2(fma2(pk2(av[2 * e], av[2 * e + 1]), cy2, pk2(V[j], V[j + 1])), V[j], V[j + 1]);
                }
            }
            if (last) {
                if (ok && rvalid) {
                    float* xr = X + (int64_t)gi * n;
                    for (int j = 0; j < 64; ++j)
                        if (128 * J + c0 + j < n) xr[128 * J + c0 + j] = V[j];
                }
            } else {
                const float vm = store_v(sb + kOwnV + rbase, rx, V, sVn,
                                         precision == LF_NS_PREC_SPLIT3 || k + 1 >= iters - 2) * (1.f / sVn);
                const float wm = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(vm)));
                if (lane == 0) atomicMax(&sh.vmax[par ^ 1u], __float_as_uint(wm));
                sV = sVn;
                fence_async_smem();
                tc_fence_before();
            }
        }
    }
    if (!ok && tid == 0) atomicExch(&g_ns_status, (int)LF_ERR_TIMEOUT);
    tc_fence_before();
    cluster_sync_all();  // no peer reads this CTA's shared memory any more
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kC256TmemCols);
    }
}

size_t tc256_smem_bytes() { return 6 * (size_t)kOpBytes + sizeof(Ns256Shared) + 1024; }

// ---------------------------------------------------------------------------
// Matrices with 128 < n <= 256 (fp32), CUDA cores.
// ---------------------------------------------------------------------------
constexpr int kMaxN = 256;
constexpr int kBigThreads = 512;

// A cluster of two CTAs per matrix; CTA r of the pair owns rows
// [r*h, min(n, (r+1)*h)), h = ceil(n/2).  The current iterate V lives in the
// output buffer (global memory, L2-resident) and the CTA's rows of the next
// iterate in shared memory; once both halves are complete (cluster barrier)
// they are written back.  Per block of 32 rows, W = V P and Y = W V are tiled
// FMA products (32-wide K chunks staged in shared memory, 4x4 outputs per
// thread): the reference 2-buffer association (V P) V.
constexpr int kBigRB = 32;   // rows per block
constexpr int kBigKC = 32;   // K chunk
constexpr int kBigCols = 256;

struct BigTile {
    float* As;  // [kBigRB][kBigKC + 1]
    float* Bs;  // [kBigKC][kBigCols]
};

// acc[4][4] += Arows[32 x n] * B[n x 256] for this thread's 4x4 tile, with
// A(i, k) and B(k, j) supplied by functors (zero outside the matrix).
template <typename FA, typename FB>
__device__ __forceinline__ void big_tile_gemm(float (&acc)[4][4], int n, const BigTile& t, FA a_at, FB b_row4) {
    const int tid = threadIdx.x;
    const int tr = tid >> 6, tc = tid & 63;  // 8 row groups x 64 column groups
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
    for (int k0 = 0; k0 < n; k0 += kBigKC) {
        __syncthreads();
        for (int e = tid; e < kBigRB * kBigKC; e += kBigThreads) {
            const int i = e / kBigKC, kk = e % kBigKC;
            t.As[i * (kBigKC + 1) + kk] = (k0 + kk < n) ? a_at(i, k0 + kk) : 0.f;
        }
        for (int e = tid; e < kBigKC * (kBigCols / 4); e += kBigThreads) {
            const int kk = e / (kBigCols / 4), j4 = e % (kBigCols / 4);
            float4 v = (k0 + kk < n) ? b_row4(k0 + kk, 4 * j4) : make_float4(0.f, 0.f, 0.f, 0.f);
            *reinterpret_cast<float4*>(&t.Bs[kk * kBigCols + 4 * j4]) = v;
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < kBigKC; ++kk) {
            const float4 b = *reinterpret_cast<const float4*>(&t.Bs[kk * kBigCols + 4 * tc]);
            float a[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = t.As[(4 * tr + i) * (kBigKC + 1) + kk];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                acc[i][0] = __fmaf_rn(a[i], b.x, acc[i][0]);
                acc[i][1] = __fmaf_rn(a[i], b.y, acc[i][1]);
                acc[i][2] = __fmaf_rn(a[i], b.z, acc[i][2]);
                acc[i][3] = __fmaf_rn(a[i], b.w, acc[i][3]);
            }
        }
    }
}

__global__ void __launch_bounds__(kBigThreads, 1)
ns_simt_big_kernel(const float* __restrict__ a, float* __restrict__ x, int n, int iters, int mode, float reg) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    cg::cluster_group cluster = cg::this_cluster();
    const int h = (n + 1) / 2;
    float* Vn = reinterpret_cast<float*>(smem_raw);        // [h][kBigCols]
    float* Wb = Vn + (size_t)h * kBigCols;                  // [kBigRB][kBigCols]
    BigTile t;
    t.As = Wb + kBigRB * kBigCols;                          // [kBigRB][kBigKC+1]
    t.Bs = t.As + kBigRB * (kBigKC + 1) + 3;                // [kBigKC][kBigCols] (16-byte aligned)
    t.Bs = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(t.Bs) + 15) & ~uintptr_t(15));
    float* red = t.Bs + kBigKC * kBigCols;                  // [kBigThreads/32]
    const int tid = threadIdx.x;
    const int rank = (int)cluster.block_rank();
    const int64_t mat = blockIdx.x / 2;
    const float* A = a + mat * (int64_t)n * n;
    float* X = x + mat * (int64_t)n * n;
    const int r_lo = rank * h, r_hi = min(n, r_lo + h);
    auto P = [&](int i, int j) -> float { return A[(int64_t)i * n + j] + (i == j ? reg : 0.f); };
    const bool vec = (n % 4) == 0;
    auto row4 = [&](const float* base, int k, int j, bool add_reg) -> float4 {
        float4 v;
        if (vec && j + 3 < n) {
            v = *reinterpret_cast<const float4*>(base + (int64_t)k * n + j);
        } else {
            v.x = j < n ? base[(int64_t)k * n + j] : 0.f;
            v.y = j + 1 < n ? base[(int64_t)k * n + j + 1] : 0.f;
            v.z = j + 2 < n ? base[(int64_t)k * n + j + 2] : 0.f;
            v.w = j + 3 < n ? base[(int64_t)k * n + j + 3] : 0.f;
        }
        if (add_reg && k >= j && k < j + 4) (&v.x)[k - j] += reg;
        return v;
    };

    float c0;
    if (mode == LF_NS_INIT_REFERENCE) {
        float mx = -1e30f;
        for (int i = tid; i < n; i += kBigThreads) {
            float s = 0.f;
            for (int j = 0; j < n; ++j) s += P(i, j);
            mx = fmaxf(mx, s);
        }
        mx = block_reduce_max<float>(mx, red);
        c0 = __fdiv_rn(1.8f, mx * mx);
    } else {
        float r1 = 0.f, ri = 0.f;
        for (int i = tid; i < n; i += kBigThreads) {
            float rs = 0.f, cs = 0.f;
            for (int j = 0; j < n; ++j) { rs += fabsf(P(i, j)); cs += fabsf(P(j, i)); }
            ri = fmaxf(ri, rs);
            r1 = fmaxf(r1, cs);
        }
        ri = block_reduce_max<float>(ri, red);
        r1 = block_reduce_max<float>(r1, red);
        c0 = __fdiv_rn(1.f, r1 * ri);
    }
    for (int e = tid; e < (r_hi - r_lo) * n; e += kBigThreads) {
        int i = r_lo + e / n, j = e % n;
        X[(int64_t)i * n + j] = (mode == LF_NS_INIT_REFERENCE ? P(i, j) : P(j, i)) * c0;
    }
    cluster.sync();

    const int tr = tid >> 6, tc = tid & 63;
    for (int it = 0; it < iters; ++it) {
        for (int r0 = r_lo; r0 < r_hi; r0 += kBigRB) {
            const int rows = min(kBigRB, r_hi - r0);
            float acc[4][4];
            // W[r0 .. r0+31, :] = V[r0 .., :] P
            big_tile_gemm(acc, n, t,
                          [&](int i, int k) { return i < rows ? X[(int64_t)(r0 + i) * n + k] : 0.f; },
                          [&](int k, int j) { return row4(A, k, j, true); });
#pragma unroll
            for (int i = 0; i < 4; ++i)
                *reinterpret_cast<float4*>(&Wb[(4 * tr + i) * kBigCols + 4 * tc]) =
                    make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
            // Y = W V;  V'[r] = 2 V[r] - Y[r]
            big_tile_gemm(acc, n, t, [&](int i, int k) { return Wb[i * kBigCols + k]; },
                          [&](int k, int j) { return row4(X, k, j, false); });
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int r = 4 * tr + i;
                if (r >= rows) continue;
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                    const int j = 4 * tc + jj;
                    if (j < n)
                        Vn[(r0 - r_lo + r) * kBigCols + j] = __fmaf_rn(2.f, X[(int64_t)(r0 + r) * n + j], -acc[i][jj]);
                }
            }
        }
        cluster.sync();  // both halves of the new iterate are complete
        for (int e = tid; e < (r_hi - r_lo) * n; e += kBigThreads) {
            int i = e / n, j = e % n;
            X[(int64_t)(r_lo + i) * n + j] = Vn[i * kBigCols + j];
        }
        cluster.sync();  // the new iterate is visible to both CTAs
    }
}

// dA = -(V^T G) V^T for any n, operands read from global memory (L2); used
// where V does not fit in shared memory.
template <typename T, typename Acc>
__global__ void __launch_bounds__(256)
ns_simt_bwd_global_kernel(const T* __restrict__ g, const T* __restrict__ v, T* __restrict__ da, int n) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int S = n + 1;
    Acc* Tr = reinterpret_cast<Acc*>(smem_raw);  // [kRB][S]
    const int tid = threadIdx.x;
    const int64_t mat = blockIdx.x;
    const T* G = g + mat * (int64_t)n * n;
    const T* V = v + mat * (int64_t)n * n;
    T* O = da + mat * (int64_t)n * n;
    const int tpr = blockDim.x / kRB;
    const int rr = tid / tpr, tj = tid - rr * tpr;
    for (int r0 = 0; r0 < n; r0 += kRB) {
        const int r = r0 + rr;
        for (int j = tj; j < n; j += tpr) {
            Acc acc = 0;
            if (r < n)
                for (int p = 0; p < n; ++p)
                    acc = fma_acc((Acc)Elem<T>::load(V[(int64_t)p * n + r]), (Acc)Elem<T>::load(G[(int64_t)p * n + j]), acc);
            Tr[rr * S + j] = acc;
        }
        __syncthreads();
        if (r < n) {
            for (int j = tj; j < n; j += tpr) {
                Acc acc = 0;
                for (int k = 0; k < n; ++k) acc = fma_acc(Tr[rr * S + k], (Acc)Elem<T>::load(V[(int64_t)j * n + k]), acc);
                O[(int64_t)r * n + j] = Elem<T>::store(-acc);
            }
        }
        __syncthreads();
    }
}

int launch_big_fwd(const void* a, void* x, int64_t batch, int64_t n, int iters, int mode, double reg,
                   cudaStream_t st) {
    const size_t h = (size_t)(n + 1) / 2;
    size_t smem = sizeof(float) * (h * kBigCols + (size_t)kBigRB * kBigCols + (size_t)kBigRB * (kBigKC + 1) + 8 +
                                   (size_t)kBigKC * kBigCols + kBigThreads / 32);
    if (smem > (size_t)max_optin_smem()) {
        set_error("NewtonInverse: n=%lld needs %zu bytes of shared memory", (long long)n, smem);
        return LF_ERR_UNSUPPORTED;
    }
    cudaFuncSetAttribute(ns_simt_big_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(2 * batch), 1, 1);
    cfg.blockDim = dim3(kBigThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t err = cudaLaunchKernelEx(&cfg, ns_simt_big_kernel, static_cast<const float*>(a), static_cast<float*>(x),
                                         (int)n, iters, mode, (float)reg);
    if (err != cudaSuccess) {
        set_error("ns_simt_big_kernel launch: %s", cudaGetErrorString(err));
        return LF_ERR_CUDA;
    }
    return check_launch("ns_simt_big_kernel");
}

int launch_tc256(const float* a, float* x, int64_t batch, int64_t n, int iters, int mode, float reg, int precision,
                 cudaStream_t st) {
    const size_t smem = tc256_smem_bytes();
    if (smem > (size_t)max_optin_smem()) {
        set_error("NewtonInverse n > 128 tensor-core path needs %zu bytes of shared memory", smem);
        return LF_ERR_UNSUPPORTED;
    }
    if (batch > 0x7fffffffLL / 4) { set_error("batch too large"); return LF_ERR_UNSUPPORTED; }
    cudaFuncSetAttribute(ns_tc256_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    ns_tc256_fwd_kernel<<<(unsigned)(4 * batch), kC256Threads, smem, st>>>(a, x, (int)n, iters, mode, reg, precision);
    return check_launch("ns_tc256_fwd_kernel");
}

template <typename T>
int launch_bwd_global(const void* g, const void* v, void* da, int64_t batch, int64_t n, cudaStream_t st) {
    using Acc = typename Elem<T>::acc;
    size_t smem = (size_t)kRB * ((size_t)n + 1) * sizeof(Acc);
    auto kern = ns_simt_bwd_global_kernel<T, Acc>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kern<<<(unsigned)batch, 256, smem, st>>>(static_cast<const T*>(g), static_cast<const T*>(v), static_cast<T*>(da), (int)n);
    return check_launch("ns_simt_bwd_global_kernel");
}

// Self-test of the bounded-wait error path: one CTA waits on an mbarrier that
// nothing arrives at; the wait gives up after `limit_ns` and the kernel
// records LF_ERR_TIMEOUT in the device status word, as the tensor-core kernel
// does, and returns normally.
__global__ void bounded_wait_probe_kernel(uint64_t limit_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) mbar_init(&bar, 1);
    __syncthreads();
    const bool ok = mbar_wait(&bar, 0, limit_ns);
    if (!ok && threadIdx.x == 0) atomicExch(&g_ns_status, (int)LF_ERR_TIMEOUT);
}

size_t tc_smem_bytes() { return 3 * (size_t)kOpBytes + sizeof(NsShared) + 1024; }


template <typename T>
int launch_tc(const T* a, T* x, int64_t batch, int64_t n, int iters, int mode, float reg, int precision,
              const float* lmk, int ld, float lscale, cudaStream_t st) {
    const size_t smem = tc_smem_bytes();
    if (smem > (size_t)max_optin_smem()) {
        set_error("NewtonInverse tensor-core path needs %zu bytes of shared memory", smem);
        return LF_ERR_UNSUPPORTED;
    }
    const int nb = tc_per_tile(n);
    const int64_t tiles = (batch + nb - 1) / nb;
    if (tiles > 0x7fffffffLL) { set_error("batch too large"); return LF_ERR_UNSUPPORTED; }
    auto kern = ns_tc_fwd_kernel<T>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    // L2 prefetch distance: the CTA slots of the device (two per SM), i.e. one wave ahead
    const int pf = lmk ? 0 : 2 * num_sms();
    kern<<<(unsigned)tiles, kTcThreads, smem, st>>>(a, x, (int)batch, (int)n, nb, iters, mode, reg, precision, lmk,
                                                    ld, lscale, pf);
    return check_launch("ns_tc_fwd_kernel");
}

template <typename T>
int launch_tc_fwd(const void* a, void* x, int64_t batch, int64_t n, int iters, int mode, float reg,
                  int precision, cudaStream_t st) {
    return launch_tc<T>(static_cast<const T*>(a), static_cast<T*>(x), batch, n, iters, mode, reg, precision,
                        nullptr, 0, 0.f, st);
}

}  // namespace
}  // namespace lfb

extern "C" int lf_laplace_newton_inverse_fwd(const void* lmk, void* x, int64_t batch, int64_t n, int64_t d,
                                             double scale, int iters, int init_mode, double reg, int precision,
                                             lf_stream_t stream) {
    using namespace lfb;
    clear_error();
    if (batch < 0 || n < 0 || d < 0) { set_error("negative size"); return LF_ERR_INVALID; }
    if (batch == 0 || n == 0) return LF_OK;
    if (!lmk || !x) { set_error("null pointer"); return LF_ERR_INVALID; }
    if (n > kTile || d < 1) {
        set_error("lf_laplace_newton_inverse_fwd supports n <= %d and d >= 1 (got n=%lld, d=%lld)", kTile,
                  (long long)n, (long long)d);
        return LF_ERR_UNSUPPORTED;
    }
    if (d > 0x7fffffffLL) { set_error("d too large"); return LF_ERR_UNSUPPORTED; }
    if (init_mode != LF_NS_INIT_REFERENCE && init_mode != LF_NS_INIT_SCALED_TRANSPOSE) {
        set_error("unknown init mode %d", init_mode);
        return LF_ERR_INVALID;
    }
    if (precision != LF_NS_PREC_SPLIT3 && precision != LF_NS_PREC_MIXED) {
        set_error("lf_laplace_newton_inverse_fwd runs on the tensor cores: precision must be split3 or mixed");
        return LF_ERR_INVALID;
    }
    if (batch > 0x7fffffff) { set_error("batch too large"); return LF_ERR_UNSUPPORTED; }
    if (iters < 0) iters = 0;
    return launch_tc<float>(nullptr, static_cast<float*>(x), batch, n, iters, init_mode, (float)reg, precision,
                            static_cast<const float*>(lmk), (int)d, (float)scale, reinterpret_cast<cudaStream_t>(stream));
}

namespace lfb {
namespace {

template <typename T>
int launch_simt_fwd(const void* a, void* x, int64_t batch, int64_t n, int iters, int mode, double reg,
                    cudaStream_t st) {
    using Acc = typename Elem<T>::acc;
    const size_t S = (size_t)n + 1;
    size_t one = (size_t)n * S * sizeof(Acc);
    size_t extra = (size_t)kRB * S * sizeof(Acc) + 8 * sizeof(Acc);
    size_t smem2 = 2 * one + extra, smem1 = one + extra;
    size_t cap = (size_t)max_optin_smem();
    if (smem2 <= cap) {
        auto kern = ns_simt_fwd_kernel<T, Acc, false>;
        if (smem2 > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem2);
        kern<<<(unsigned)batch, 256, smem2, st>>>(static_cast<const T*>(a), static_cast<T*>(x), (int)n, iters, mode, (Acc)reg);
        return check_launch("ns_simt_fwd_kernel");
    }
    if constexpr (sizeof(T) == sizeof(Acc)) {
        if (smem1 <= cap) {
            auto kern = ns_simt_fwd_kernel<T, Acc, true>;
            if (smem1 > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem1);
            kern<<<(unsigned)batch, 256, smem1, st>>>(static_cast<const T*>(a), static_cast<T*>(x), (int)n, iters, mode, (Acc)reg);
            return check_launch("ns_simt_fwd_kernel");
        }
    }
    set_error("NewtonInverse: n=%lld does not fit in shared memory", (long long)n);
    return LF_ERR_UNSUPPORTED;
}

template <typename T>
int launch_simt_bwd(const void* g, const void* v, void* da, int64_t batch, int64_t n, cudaStream_t st) {
    using Acc = typename Elem<T>::acc;
    const size_t S = (size_t)n + 1;
    size_t smem = ((size_t)n * S + (size_t)kRB * S) * sizeof(Acc);
    if (smem > (size_t)max_optin_smem()) {
        set_error("NewtonInverse backward: n=%lld does not fit in shared memory", (long long)n);
        return LF_ERR_UNSUPPORTED;
    }
    auto kern = ns_simt_bwd_kernel<T, Acc>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kern<<<(unsigned)batch, 256, smem, st>>>(static_cast<const T*>(g), static_cast<const T*>(v), static_cast<T*>(da), (int)n);
    return check_launch("ns_simt_bwd_kernel");
}

int check_ns(const void* a, const void* x, int64_t batch, int64_t n, int dtype) {
    if (dtype_size(dtype) == 0) { set_error("unsupported dtype code %d", dtype); return LF_ERR_DTYPE; }
    if (batch < 0 || n < 0) { set_error("negative size"); return LF_ERR_INVALID; }
    if (batch > 0x7fffffffLL) { set_error("batch too large"); return LF_ERR_UNSUPPORTED; }
    if (n > kMaxN) { set_error("NewtonInverse supports n <= %d (got %lld)", kMaxN, (long long)n); return LF_ERR_UNSUPPORTED; }
    if (batch > 0 && n > 0 && (!a || !x)) { set_error("null pointer"); return LF_ERR_INVALID; }
    return LF_OK;
}

}  // namespace
}  // namespace lfb

using namespace lfb;

extern "C" int lf_newton_inverse_supported(int64_t n) { return (n >= 1 && n <= kMaxN) ? 1 : 0; }

extern "C" int lf_newton_inverse_fwd_ex(const void* a, void* x, int64_t batch, int64_t n, int iters,
                                        int dtype, int init_mode, double reg, int precision,
                                        lf_stream_t stream) {
    clear_error();
    int rc = check_ns(a, x, batch, n, dtype);
    if (rc) return rc;
    if (init_mode != LF_NS_INIT_REFERENCE && init_mode != LF_NS_INIT_SCALED_TRANSPOSE) {
        set_error("unknown init mode %d", init_mode);
        return LF_ERR_INVALID;
    }
    if (precision < LF_NS_PREC_SPLIT3 || precision > LF_NS_PREC_FP32_SIMT) {
        set_error("unknown precision %d", precision);
        return LF_ERR_INVALID;
    }
    if (batch == 0 || n == 0) return LF_OK;
    if (iters < 0) iters = 0;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (n > kTile) {
        if (dtype != LF_F32) {
            set_error("NewtonInverse: n=%lld > %d is supported for fp32 only", (long long)n, kTile);
            return LF_ERR_UNSUPPORTED;
        }
        if (precision == LF_NS_PREC_FP32_SIMT) return launch_big_fwd(a, x, batch, n, iters, init_mode, reg, st);
        return launch_tc256(static_cast<const float*>(a), static_cast<float*>(x), batch, n, iters, init_mode,
                            (float)reg, precision, st);
    }
    if (dtype == LF_F64) return launch_simt_fwd<double>(a, x, batch, n, iters, init_mode, reg, st);
    if (precision == LF_NS_PREC_FP32_SIMT) {
        LF_DISPATCH(dtype, T, return launch_simt_fwd<T>(a, x, batch, n, iters, init_mode, reg, st));
    }
    switch (dtype) {
        case LF_F32: return launch_tc_fwd<float>(a, x, batch, n, iters, init_mode, (float)reg, precision, st);
        case LF_F16: return launch_tc_fwd<__half>(a, x, batch, n, iters, init_mode, (float)reg, precision, st);
        case LF_BF16: return launch_tc_fwd<__nv_bfloat16>(a, x, batch, n, iters, init_mode, (float)reg, precision, st);
        default: break;
    }
    set_error("unsupported dtype code %d", dtype);
    return LF_ERR_DTYPE;
}

extern "C" int lf_newton_inverse_fwd(const void* a, void* x, int64_t batch, int64_t n, int iters, int dtype,
                                     lf_stream_t stream) {
    return lf_newton_inverse_fwd_ex(a, x, batch, n, iters, dtype, LF_NS_INIT_REFERENCE, 0.01,
                                    LF_NS_PREC_SPLIT3, stream);
}

extern "C" int lf_newton_inverse_bwd(const void* g, const void* v, void* da, int64_t batch, int64_t n, int dtype,
                                     lf_stream_t stream) {
    clear_error();
    int rc = check_ns(g, v, batch, n, dtype);
    if (rc) return rc;
    if (!da && batch * n > 0) { set_error("null grad_mat"); return LF_ERR_INVALID; }
    if (batch == 0 || n == 0) return LF_OK;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (n > kTile) { LF_DISPATCH(dtype, T, return launch_bwd_global<T>(g, v, da, batch, n, st)); }
    switch (dtype) {  // tensor cores for fp32 / fp16 / bf16; fp64 on CUDA cores
        case LF_F32: return launch_tc_bwd<float>(g, v, da, batch, n, st);
        case LF_F16: return launch_tc_bwd<__half>(g, v, da, batch, n, st);
        case LF_BF16: return launch_tc_bwd<__nv_bfloat16>(g, v, da, batch, n, st);
        default: break;
    }
    LF_DISPATCH(dtype, T, return launch_simt_bwd<T>(g, v, da, batch, n, st));
    return LF_OK;
}

extern "C" int lf_newton_inverse_residual(const void* a, const void* x, void* res, int64_t batch, int64_t n,
                                          double reg, int dtype, lf_stream_t stream) {
    clear_error();
    int rc = check_ns(a, x, batch, n, dtype);
    if (rc) return rc;
    if (!res && batch > 0) { set_error("null residual output"); return LF_ERR_INVALID; }
    if (batch == 0) return LF_OK;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (n == 0) {
        if (cudaMemsetAsync(res, 0, (size_t)batch * (dtype == LF_F64 ? 8 : 4), st) != cudaSuccess) return check_launch("memset");
        return LF_OK;
    }
    LF_DISPATCH(dtype, T, {
        using Acc = typename Elem<T>::acc;
        ns_residual_kernel<T, Acc><<<(unsigned)batch, 256, 0, st>>>(static_cast<const T*>(a), static_cast<const T*>(x),
                                                                    static_cast<Acc*>(res), (int)n, (Acc)reg);
        return check_launch("ns_residual_kernel");
    });
    return LF_OK;
}

extern "C" int lf_selftest_bounded_wait(int timeout_ms, lf_stream_t stream) {
    clear_error();
    if (timeout_ms < 1 || timeout_ms > 10000) { set_error("timeout_ms must be in [1, 10000]"); return LF_ERR_INVALID; }
    bounded_wait_probe_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>((uint64_t)timeout_ms * 1000000ull);
    return check_launch("bounded_wait_probe_kernel");
}

// Synchronises the current device and returns (and optionally clears) the
// status word set by kernels whose bounded waits expired.
extern "C" int lf_device_status(int clear) {
    clear_error();
    if (cudaDeviceSynchronize() != cudaSuccess) return check_launch("cudaDeviceSynchronize");
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_ns_status, sizeof(int)) != cudaSuccess) return check_launch("status read");
    if (clear && v) {
        int z = 0;
        if (cudaMemcpyToSymbol(g_ns_status, &z, sizeof(int)) != cudaSuccess) return check_launch("status clear");
    }
    const int pv = peer_status(clear != 0);  // the peer barrier's word
    return v ? v : pv;
}

