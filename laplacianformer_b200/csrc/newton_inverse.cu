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

// Phase timestamps of CTA 0 for kernel development builds (-DLF_NS_TRACE);
// compiled out otherwise.
#ifdef LF_NS_TRACE
__device__ long long g_ns_trace[16][32];
#define NS_TRACE(it, k)                                                                          \
    do {                                                                                         \
        if (blockIdx.x == 0 && (threadIdx.x == 0 || threadIdx.x == 256) && (it) < 16)            \
            g_ns_trace[it][(k) + (threadIdx.x ? 16 : 0)] = clock64();                            \
    } while (0)
#else
#define NS_TRACE(it, k) \
    do {                \
    } while (0)
#endif

namespace {

constexpr int kNsThreads = 512;
constexpr int kTile = 128;                 // padded matrix size
constexpr int kOpBytes = kTile * kTile * 2; // one fp16 operand (32 KB)
constexpr bool kWInTmem = true;        // W operand of the second product in TMEM (else shared memory)
constexpr bool kSplitW = false;        // W = V P as two N = 64 halves (true) or one N = 128 product
constexpr int kTmemCols = 512;             // W and Y accumulators + fp32 V (384 used)

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
// reports LF_ERR_TIMEOUT instead of hanging the GPU).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns = 2000000000ull) {
    const uint32_t addr = smem_u32(bar);
    const uint64_t t0 = global_ns();
    for (uint32_t spin = 0;; ++spin) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}\n"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
        if ((spin & 255u) == 255u && global_ns() - t0 > limit_ns) return false;
    }
}

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

// D[tmem] (+)= A[smem] * B[smem], kind::f16, cta_group::1.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem], kind::f16: A is 128 lanes (rows) x K fp16
// with consecutive K pairs packed in one 32-bit column.
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets lane
// (quadrant*32 + i), columns [col, col+32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t* r = reinterpret_cast<uint32_t*>(v);
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
    const uint32_t* r = reinterpret_cast<const uint32_t*>(v);
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
        "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
        "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// Ties registers written by tcgen05.ld to a point after tcgen05.wait::ld so
// that the compiler cannot hoist their uses above the wait.
__device__ __forceinline__ void reg_fence(float (&v)[32]) {
#pragma unroll
    for (int i = 0; i < 32; ++i) asm volatile("" : "+f"(v[i]));
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------------------
// Operand layout: a 128x128 fp16 matrix X[r][c], row-major with the 128-byte
// swizzle.  Columns [0,64) and [64,128) form two 16 KB blocks; row r of a
// block is 128 bytes at r*128 and its 16-byte chunk k sits at chunk k^(r%8).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t op_chunk_offset(int r, int col8) {
    // byte offset of the 16-byte chunk holding columns [8*col8, 8*col8+8) of row r
    return (uint32_t)((col8 >> 3) * 16384 + r * 128 + (((col8 & 7) ^ (r & 7)) << 4));
}

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
// A operand (K-major view of the row-major layout), K step ks of 16 columns.
__device__ __forceinline__ uint64_t desc_a(uint32_t base, int ks) {
    return make_desc(base + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024);
}
// B operand (MN-major view: rows = k, contiguous columns = n), K step ks.
__device__ __forceinline__ uint64_t desc_b(uint32_t base, int ks) {
    return make_desc(base + ks * 2048, 16384, 1024);
}
// Power-of-two scale that maps max|x| into [2^14, 2^15); 1 for 0 or non-finite.
__device__ __forceinline__ float split_scale(float mx) {
    if (!(mx > 0.f) || !isfinite(mx)) return 1.f;
    int e;
    frexpf(mx, &e);  // mx = f * 2^e, f in [0.5, 1)
    return ldexpf(1.f, 15 - e);
}

__device__ __forceinline__ void split_store(unsigned char* hi_base, unsigned char* lo_base, int r,
                                            int col0, const float (&v)[32], float s) {
    // v holds columns [col0, col0+32) of row r (col0 a multiple of 32); stores
    // hi = fp16(v*s) and lo = fp16(v*s - hi), two elements per conversion.
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        uint32_t h[4], l[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 xs = make_float2(v[8 * k + 2 * e] * s, v[8 * k + 2 * e + 1] * s);
            const __half2 hh = __float22half2_rn(xs);
            const float2 hb = __half22float2(hh);
            const __half2 ll = __float22half2_rn(make_float2(xs.x - hb.x, xs.y - hb.y));
            h[e] = *reinterpret_cast<const uint32_t*>(&hh);
            l[e] = *reinterpret_cast<const uint32_t*>(&ll);
        }
        uint32_t off = op_chunk_offset(r, (col0 >> 3) + k);
        *reinterpret_cast<uint4*>(hi_base + off) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4*>(lo_base + off) = make_uint4(l[0], l[1], l[2], l[3]);
    }
}

__device__ __forceinline__ void named_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void named_arrive(int id, int count) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// hi/lo fp16 split of 32 values into packed pairs (element 2i in the low half).
__device__ __forceinline__ void split_pack(const float (&v)[32], float s, uint32_t (&h)[16], uint32_t (&l)[16]) {
#pragma unroll
    for (int e = 0; e < 16; ++e) {
        const float2 xs = make_float2(v[2 * e] * s, v[2 * e + 1] * s);
        const __half2 hh = __float22half2_rn(xs);
        const float2 hb = __half22float2(hh);
        const __half2 ll = __float22half2_rn(make_float2(xs.x - hb.x, xs.y - hb.y));
        h[e] = *reinterpret_cast<const uint32_t*>(&hh);
        l[e] = *reinterpret_cast<const uint32_t*>(&ll);
    }
}

// Y += W * V for K steps [ks0, ks1) with W (hi at a_hi, lo at a_lo) in TMEM.
__device__ __forceinline__ void issue_mma_ts(uint32_t acc, uint32_t a_hi, uint32_t a_lo, uint32_t b_hi,
                                             uint32_t b_lo, int ks0, int ks1, int nterm, bool first) {
    constexpr uint32_t idesc = (1u << 4) | (1u << 16) | ((uint32_t)(kTile >> 3) << 17) | ((uint32_t)(kTile >> 4) << 24);
    for (int ks = ks0; ks < ks1; ++ks) {
        mma_f16_ts(acc, a_hi + ks * 8, desc_b(b_hi, ks), idesc, (first && ks == ks0) ? 0u : 1u);
        if (nterm == 3) {
            mma_f16_ts(acc, a_hi + ks * 8, desc_b(b_lo, ks), idesc, 1u);
            mma_f16_ts(acc, a_lo + ks * 8, desc_b(b_hi, ks), idesc, 1u);
        }
    }
}

struct NsShared {
    uint64_t bar[3];            // W columns [0,64), W columns [64,128), Y
    uint32_t tmem_base;
    float red[kNsThreads / 32][4];
    float colsum[kTile];
};

// One K-range of a product into the accumulator: N columns (64 or 128),
// nterm = 1 (hi*hi) or 3 (hi*hi + hi*lo + lo*hi).  b_* may point into the
// second 64-column block for an N = 64 product.
template <int N>
__device__ __forceinline__ void issue_mma(uint32_t acc, uint32_t a_hi, uint32_t a_lo, uint32_t b_hi,
                                          uint32_t b_lo, int ks0, int ks1, int nterm, bool first) {
    constexpr uint32_t idesc = (1u << 4) | (1u << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(kTile >> 4) << 24);
    for (int ks = ks0; ks < ks1; ++ks) {
        mma_f16(acc, desc_a(a_hi, ks), desc_b(b_hi, ks), idesc, (first && ks == ks0) ? 0u : 1u);
        if (nterm == 3) {
            mma_f16(acc, desc_a(a_hi, ks), desc_b(b_lo, ks), idesc, 1u);
            mma_f16(acc, desc_a(a_lo, ks), desc_b(b_hi, ks), idesc, 1u);
        }
    }
}

// Block-wide max of four values (two __syncthreads).
__device__ __forceinline__ void block_max4(float (&v)[4], NsShared& sh) {
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v[k] = fmaxf(v[k], __shfl_xor_sync(0xffffffffu, v[k], o));
    const int warp = threadIdx.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0)
#pragma unroll
        for (int k = 0; k < 4; ++k) sh.red[warp][k] = v[k];
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        float m = sh.red[0][k];
        for (int w = 1; w < kNsThreads / 32; ++w) m = fmaxf(m, sh.red[w][k]);
        v[k] = m;
    }
}

// Set-up staging tile: 128x128 fp32, element (i, c) at i*128 + swz(i, c).
// The XOR keeps row writes (lanes over c) and column reads (lanes over i)
// free of bank conflicts.
__device__ __forceinline__ int stage_idx(int i, int c) { return i * kTile + (c ^ (i & 31) ^ ((c >> 5) & 3)); }

// grid = batch, block = 512 threads (16 warps).  Warp w owns TMEM lanes
// 32*(w%4).. (matrix rows) and the 32 columns 32*(w/4).. of the tile.
//
// Per iteration, with one thread issuing every MMA:
//   W[:, 0:64]  = V P[:, 0:64]   -> bar[0]   (warps of column groups 0,1 convert it)
//   W[:, 64:128]= V P[:, 64:128] -> bar[1]   (column groups 2,3), overlapping the first conversion
//   Y  = W[:, 0:64] V[0:64, :]   issued as soon as groups 0,1 have stored their half of W,
//      + W[:, 64:128] V[64:128,:] issued when groups 2,3 have     -> bar[2]
//   V <- 2V - Y (all warps), new split scale from a block max.
// W's split scale comes from the bound max|W| <= ||V||_inf * max|P| (known
// before the product; ||V||_inf exactly for V0, then n * max|V|), so its
// conversion needs no reduction.  A loose bound only lowers the magnitude of
// the scaled values; fp16 keeps 11 significant bits down to 2^-14.
template <typename T>
__global__ void __launch_bounds__(kNsThreads, 1)
ns_tc_fwd_kernel(const T* __restrict__ a, T* __restrict__ x, int n, int iters, int mode, float reg,
                 int precision, const float* __restrict__ lmk, int ld, float lscale) {
    extern __shared__ __align__(16) unsigned char smem_raw[];  // re-aligned to 1024 below
    unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* Ph = base;
    unsigned char* Pl = base + 1 * kOpBytes;
    unsigned char* Vh = base + 2 * kOpBytes;
    unsigned char* Vl = base + 3 * kOpBytes;
    unsigned char* Wh = base + 4 * kOpBytes;
    unsigned char* Wl = base + 5 * kOpBytes;
    float* stage = reinterpret_cast<float*>(Wh);  // 128x128 fp32 during set-up (spans Wh and Wl)
    NsShared& sh = *reinterpret_cast<NsShared*>(base + 6 * kOpBytes);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quad = warp & 3, cg = warp >> 2;
    const int row = quad * 32 + lane;  // matrix row this thread owns in the epilogues
    const int col0 = cg * 32;          // its 32 columns
    const int64_t mat = blockIdx.x;
    const T* A = a + mat * (int64_t)n * n;
    T* X = x + mat * (int64_t)n * n;

    if (tid == 0) {
        for (int b = 0; b < 3; ++b) mbar_init(&sh.bar[b], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (tid < kTile) sh.colsum[tid] = 0.f;
    if (warp == 0) tmem_alloc(&sh.tmem_base, kTmemCols);
    __syncthreads();

    // ---- optional: A from landmarks -------------------------------------------
    // With lmk != nullptr, A[i][c] = exp(lscale * sum_k |L[i][k] - L[c][k]|)
    // is formed here (the channel sum in order with the LaplaceSub forward's
    // fp32 operations, so A is bit-identical to lf_laplace_kernel_fwd(L, L^T)).
    // L^T of this matrix is staged as LT[k][c] in the Vh/Vl region (free until
    // V0 is written after the set-up): row i is a warp-uniform broadcast and a
    // lane's four columns one 16-byte load.
    float* LT = reinterpret_cast<float*>(Vh);
    if (lmk) {
        const float* Lb = lmk + mat * (int64_t)n * ld;
        for (int e = tid; e < ld * kTile; e += kNsThreads) {
            const int c = e / ld, k = e - c * ld;  // coalesced read of L[c][k]
            LT[k * kTile + c] = (c < n) ? Lb[(int64_t)c * ld + k] : 0.f;
        }
        __syncthreads();
    }

    // ---- set-up: P = A + reg I into the staging tile -------------------------
    // Warp w loads rows w, w+16, ...; lane l holds columns 4l..4l+3.
    float mx[4] = {-1e30f, 0.f, 0.f, 0.f};  // signed row sum, |row| sum, max|P|, |col| sum
    float colacc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int i = warp; i < kTile; i += kNsThreads / 32) {
        float v[4];
        float lsum[4] = {0.f, 0.f, 0.f, 0.f};
        if (lmk && i < n) {
            for (int k = 0; k < ld; ++k) {
                const float li = LT[k * kTile + i];
                const float4 lc = *reinterpret_cast<const float4*>(LT + k * kTile + 4 * lane);
                lsum[0] = add_abs_ftz(lsum[0], sub_ftz(li, lc.x));
                lsum[1] = add_abs_ftz(lsum[1], sub_ftz(li, lc.y));
                lsum[2] = add_abs_ftz(lsum[2], sub_ftz(li, lc.z));
                lsum[3] = add_abs_ftz(lsum[3], sub_ftz(li, lc.w));
            }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            int c = 4 * lane + e;
            float t = 0.f;
            if (i < n && c < n) {
                const float av = lmk ? expf(lscale * lsum[e]) : Elem<T>::load(A[(int64_t)i * n + c]);
                t = av + (i == c ? reg : 0.f);
            }
            v[e] = t;
            stage[stage_idx(i, c)] = t;
            colacc[e] += fabsf(t);
            mx[2] = fmaxf(mx[2], fabsf(t));
        }
        float rs = (v[0] + v[1]) + (v[2] + v[3]);
        float ra = (fabsf(v[0]) + fabsf(v[1])) + (fabsf(v[2]) + fabsf(v[3]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            rs += __shfl_xor_sync(0xffffffffu, rs, o);
            ra += __shfl_xor_sync(0xffffffffu, ra, o);
        }
        if (i < n) {
            mx[0] = fmaxf(mx[0], rs);
            mx[1] = fmaxf(mx[1], ra);
        }
    }
    // column |sums|: per-warp partials combined in warp order (deterministic,
    // so equal inputs give equal bits); Ph is free until P is split below
    float* cpart = reinterpret_cast<float*>(Ph);  // [16 warps][kTile]
#pragma unroll
    for (int e = 0; e < 4; ++e) cpart[warp * kTile + 4 * lane + e] = colacc[e];
    __syncthreads();
    if (tid < kTile) {
        float cs = 0.f;
        for (int w = 0; w < kNsThreads / 32; ++w) cs += cpart[w * kTile + tid];
        mx[3] = cs;
    }
    block_max4(mx, sh);
    const float pmax = mx[2];
    const float v0_scale = (mode == LF_NS_INIT_REFERENCE) ? __fdiv_rn(1.8f, mx[0] * mx[0])
                                                         : __fdiv_rn(1.0f, mx[3] * mx[1]);
    const float sP = split_scale(pmax);
    float sV = split_scale(pmax * fabsf(v0_scale));
    // ||V0||_inf: alpha*||P||_inf, or c*||P||_1 for V0 = c P^T.
    float vinf = fabsf(v0_scale) * (mode == LF_NS_INIT_REFERENCE ? mx[1] : mx[3]);

    tc_fence_after();
    const uint32_t tmem = sh.tmem_base;
    const uint32_t t_lane = (uint32_t)(quad * 32) << 16;
    const uint32_t t_w = tmem + t_lane;              // W accumulator, columns [0,128)
    const uint32_t t_y = tmem + t_lane + kTile;      // Y accumulator, columns [128,256)
    const uint32_t t_v = tmem + t_lane + 2 * kTile;  // fp32 V, columns [256,384)
    const uint32_t t_wa = tmem + t_lane + 3 * kTile;  // W hi [384,448) and lo [448,512), fp16 pairs
    const uint32_t a_whi = tmem + 3 * kTile, a_wlo = tmem + 3 * kTile + kTile / 2;  // as MMA A operands
    {
        float pv[32], vv[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
            int c = col0 + e;
            pv[e] = stage[stage_idx(row, c)];
            float src = (mode == LF_NS_INIT_REFERENCE) ? pv[e] : stage[stage_idx(c, row)];
            vv[e] = src * v0_scale;
        }
        split_store(Ph, Pl, row, col0, pv, sP);
        if (iters > 0) {
            split_store(Vh, Vl, row, col0, vv, sV);
            tmem_st32(t_v + col0, vv);
            tmem_wait_st();
        } else if (row < n) {
#pragma unroll
            for (int e = 0; e < 32; ++e)
                if (col0 + e < n) X[(int64_t)row * n + col0 + e] = Elem<T>::store(vv[e]);
        }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();  // staging reads done before W is overwritten; operands visible

    const uint32_t aPh = smem_u32(Ph), aPl = smem_u32(Pl), aVh = smem_u32(Vh), aVl = smem_u32(Vl);
    const uint32_t aWh = smem_u32(Wh), aWl = smem_u32(Wl);
    uint32_t phase = 0;
    bool ok = true;

    for (int it = 0; it < iters; ++it) {
        const int nterm = (precision == LF_NS_PREC_MIXED && it < iters - 2) ? 1 : 3;
        const bool last = (it == iters - 1);
        const float sW = split_scale(vinf * pmax);
        NS_TRACE(it, 0);
        // ---- W = V P in two column halves ---------------------------------
        if (tid == 0) {
            tc_fence_after();
            if (kSplitW) {
                issue_mma<64>(tmem, aVh, aVl, aPh, aPl, 0, kTile / 16, nterm, true);
                mma_commit(&sh.bar[0]);
                issue_mma<64>(tmem + 64, aVh, aVl, aPh + 16384, aPl + 16384, 0, kTile / 16, nterm, true);
                mma_commit(&sh.bar[1]);
            } else {
                // one N = 128 product reads each A tile once (M = 128 MMAs with
                // both operands in shared memory are bound by its bandwidth)
                issue_mma<128>(tmem, aVh, aVl, aPh, aPl, 0, kTile / 16, nterm, true);
                mma_commit(&sh.bar[0]);
                mma_commit(&sh.bar[1]);
            }
        }
        NS_TRACE(it, 1);
        const bool lo_half = cg < 2;
        bool okw = mbar_wait(&sh.bar[lo_half ? 0 : 1], phase);
        NS_TRACE(it, 2);
        tc_fence_after();
        {
            float wv[32];
            tmem_ld32(t_w + col0, wv);
            tmem_wait_ld();
            reg_fence(wv);
            NS_TRACE(it, 12);
            // acc = W * sV * sP; the stored operand is W * sW (all powers of two)
            if (kWInTmem) {
                uint32_t hp[16], lp[16];
                split_pack(wv, sW * (1.f / sV) * (1.f / sP), hp, lp);
                tmem_st16(t_wa + col0 / 2, hp);
                tmem_st16(t_wa + kTile / 2 + col0 / 2, lp);
                tmem_wait_st();
            } else {
                split_store(Wh, Wl, row, col0, wv, sW * (1.f / sV) * (1.f / sP));
            }
        }
        NS_TRACE(it, 3);
        fence_async_smem();
        tc_fence_before();
        // ---- Y = W V, K split so that the first half starts early ----------
        if (lo_half) {
            named_sync(1, kNsThreads / 2);
            if (tid == 0) {
                tc_fence_after();
                if (kWInTmem) issue_mma_ts(tmem + kTile, a_whi, a_wlo, aVh, aVl, 0, kTile / 32, nterm, true);
                else issue_mma<128>(tmem + kTile, aWh, aWl, aVh, aVl, 0, kTile / 32, nterm, true);
            }
            if (warp == 0) {
                named_sync(2, kNsThreads / 2 + 32);
                if (lane == 0) {
                    tc_fence_after();
                    if (kWInTmem) issue_mma_ts(tmem + kTile, a_whi, a_wlo, aVh, aVl, kTile / 32, kTile / 16, nterm, false);
                    else issue_mma<128>(tmem + kTile, aWh, aWl, aVh, aVl, kTile / 32, kTile / 16, nterm, false);
                    mma_commit(&sh.bar[2]);
                }
                __syncwarp();
            }
        } else {
            named_arrive(2, kNsThreads / 2 + 32);
        }
        NS_TRACE(it, 4);
        okw = mbar_wait(&sh.bar[2], phase) && okw;
        NS_TRACE(it, 5);
        phase ^= 1;
        ok = !__syncthreads_or(!okw);
        if (!ok) break;
        tc_fence_after();
        // ---- V <- 2V - Y ----------------------------------------------------
        float vn[32];
        float lmax = 0.f;
        {
            float yv[32];
            tmem_ld32(t_y + col0, yv);
            tmem_ld32(t_v + col0, vn);
            tmem_wait_ld();
            reg_fence(yv);
            reg_fence(vn);
            NS_TRACE(it, 9);
            const float c2 = (1.f / sW) * (1.f / sV);  // acc = Y * sW * sV
#pragma unroll
            for (int e = 0; e < 32; ++e) {
                vn[e] = fmaf(yv[e], -c2, 2.f * vn[e]);
                lmax = fmaxf(lmax, fabsf(vn[e]));
            }
        }
        if (last) {
            if (row < n) {
#pragma unroll
                for (int e = 0; e < 32; ++e)
                    if (col0 + e < n) X[(int64_t)row * n + col0 + e] = Elem<T>::store(vn[e]);
            }
            break;
        }
        NS_TRACE(it, 10);
        tmem_st32(t_v + col0, vn);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
        if (lane == 0) sh.red[warp][0] = lmax;
        __syncthreads();
        NS_TRACE(it, 11);
        float m = sh.red[0][0];
        for (int w = 1; w < kNsThreads / 32; ++w) m = fmaxf(m, sh.red[w][0]);
        sV = split_scale(m);
        vinf = (float)n * m;  // ||V||_inf <= n * max|V|
        split_store(Vh, Vl, row, col0, vn, sV);
        NS_TRACE(it, 7);
        tmem_wait_st();
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        NS_TRACE(it, 8);
    }
    if (!ok && tid == 0) atomicExch(&g_ns_status, (int)LF_ERR_TIMEOUT);
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

size_t tc_smem_bytes() { return 6 * (size_t)kOpBytes + sizeof(NsShared) + 1024; }

template <typename T>
int launch_tc_fwd(const void* a, void* x, int64_t batch, int64_t n, int iters, int mode, float reg,
                  int precision, cudaStream_t st) {
    size_t smem = tc_smem_bytes();
    if (smem > (size_t)max_optin_smem()) {
        set_error("NewtonInverse tensor-core path needs %zu bytes of shared memory", smem);
        return LF_ERR_UNSUPPORTED;
    }
    auto kern = ns_tc_fwd_kernel<T>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kern<<<(unsigned)batch, kNsThreads, smem, st>>>(static_cast<const T*>(a), static_cast<T*>(x), (int)n, iters,
                                                    mode, reg, precision, nullptr, 0, 0.f);
    return check_launch("ns_tc_fwd_kernel");
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
    if (n > kTile || d < 1 || d * kTile * 4 > 2 * kOpBytes) {
        set_error("lf_laplace_newton_inverse_fwd supports n <= %d and 1 <= d <= %d (got n=%lld, d=%lld)", kTile,
                  2 * kOpBytes / (kTile * 4), (long long)n, (long long)d);
        return LF_ERR_UNSUPPORTED;
    }
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
    const size_t smem = tc_smem_bytes();
    if (smem > (size_t)max_optin_smem()) {
        set_error("NewtonInverse tensor-core path needs %zu bytes of shared memory", smem);
        return LF_ERR_UNSUPPORTED;
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    auto kern = ns_tc_fwd_kernel<float>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kern<<<(unsigned)batch, kNsThreads, smem, st>>>(nullptr, static_cast<float*>(x), (int)n, iters, init_mode,
                                                    (float)reg, precision, static_cast<const float*>(lmk), (int)d,
                                                    (float)scale);
    return check_launch("ns_tc_fwd_kernel");
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
        return launch_big_fwd(a, x, batch, n, iters, init_mode, reg, st);
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
    return v;
}

#ifdef LF_NS_TRACE
extern "C" LF_API int lf_ns_trace_read(long long* out) {
    return cudaMemcpyFromSymbol(out, g_ns_trace, sizeof(long long) * 16 * 32) == cudaSuccess ? 0 : 1;
}
#endif
