// LaplaceSubtraction on B200 (sm_100a): pairwise L1 distance between queries
// and landmarks, its two gradients, and the reference's legacy reduce path.
//
//   S[b,i,j]   = sum_c |Q[b,i,c] - KT[b,c,j]|                (forward)
//   dQ[b,i,c]  =  sum_j G[b,i,j] * sign(Q[b,i,c] - KT[b,c,j])  (backward, query)
//   dKT[b,c,j] = -sum_i G[b,i,j] * sign(Q[b,i,c] - KT[b,c,j])  (backward, key)
//
// Semantics follow src/LaplaceSubtraction_cuda_kernel.cu of the reference
// (forward :47-141, backward-query :148-267, backward-key :274-393, reduce
// :399-447).  An L1 distance is not a contraction, so these kernels run on
// the CUDA cores; the design targets the FP32 issue rate and HBM:
//
// * Forward: lanes own query rows, a thread keeps TM rows x 16 channels of
//   Q in registers and a chunk of MC landmarks' accumulators; landmark values
//   are warp-uniform broadcasts from shared memory (one 128-bit LDS per four
//   channels).  Each output is accumulated over the channels in order, with
//   the same fp32 operations as the reference, so fp32/fp64 results are
//   bit-identical to the reference kernel.
// * Backward (fused): lanes own channels, a warp walks query rows and keeps
//   KT[c, j] and the dKT partials of its chunk of landmarks in registers, so
//   both reductions are thread-local.  sign(q-k)*g costs one FFMA.SAT
//   (t = sat(d*2^125 + 0.5) in {0, 1/2, 1}, sign = 2t - 1 exactly):
//       dQ  = sum_j 2g*t - sum_j g,    dKT = sum_i g - sum_i 2g*t.
//   The CTAs that split one (b,h) along the rows form a thread-block cluster
//   and add their dKT partials through distributed shared memory; no atomics
//   in global memory and no pre-zeroed output.
#include <cooperative_groups.h>
#include <stdlib.h>

#include <map>
#include <mutex>
#include <tuple>

#include "lf_common.cuh"

namespace cg = cooperative_groups;

namespace lfb {
namespace {

constexpr int kThreads = 256;

// Fraction of the machine's CTA slots that `total` CTAs keep busy over the
// waves they need (1.0 = no partial last wave).
inline double wave_efficiency(int64_t total, int64_t slots) {
    if (total <= 0 || slots <= 0) return 0.0;
    int64_t waves = (total + slots - 1) / slots;
    return (double)total / (double)(waves * slots);
}

template <typename K>
int64_t cta_slots(K kern, size_t smem, int threads = kThreads) {
    // The occupancy query costs microseconds of host time per launch, so the
    // answer is cached per (kernel, device, shared-memory size).  Launchers
    // that compare two kernels query both on every call, so the cache keeps
    // every key rather than only the last one.
    static std::mutex mu;
    static std::map<std::tuple<const void*, int, size_t, int>, int> cache;
    int dev = 0;
    cudaGetDevice(&dev);
    const auto key = std::make_tuple(reinterpret_cast<const void*>(kern), dev, smem, threads);
    {
        std::lock_guard<std::mutex> lock(mu);
        auto it = cache.find(key);
        if (it != cache.end()) return (int64_t)it->second * num_sms();
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem) != cudaSuccess || per_sm < 1)
        per_sm = 1;
    std::lock_guard<std::mutex> lock(mu);
    cache[key] = per_sm;
    return (int64_t)per_sm * num_sms();
}

// Clusters of `csize` CTAs (`threads` threads, `smem` bytes each) that the
// current device runs at once (0: the size does not fit); cached like
// cta_slots.
template <typename K>
int active_clusters(K kern, int csize, int threads, size_t smem) {
    static std::mutex mu;
    static std::map<std::tuple<const void*, int, size_t, int, int>, int> cache;
    int dev = 0;
    cudaGetDevice(&dev);
    const auto key = std::make_tuple(reinterpret_cast<const void*>(kern), dev, smem, threads, csize);
    {
        std::lock_guard<std::mutex> lock(mu);
        auto it = cache.find(key);
        if (it != cache.end()) return it->second;
    }
    cudaLaunchConfig_t probe = {};
    probe.gridDim = dim3((unsigned)csize, 1, 1);
    probe.blockDim = dim3((unsigned)threads, 1, 1);
    probe.dynamicSmemBytes = smem;
    cudaLaunchAttribute pa[1];
    pa[0].id = cudaLaunchAttributeClusterDimension;
    pa[0].val.clusterDim.x = (unsigned)csize;
    pa[0].val.clusterDim.y = 1;
    pa[0].val.clusterDim.z = 1;
    probe.attrs = pa;
    probe.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &probe) != cudaSuccess) {
        cudaGetLastError();
        clusters = 0;
    }
    std::lock_guard<std::mutex> lock(mu);
    cache[key] = clusters;
    return clusters;
}

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ void load_chunk16(const T* __restrict__ src, int valid, bool vec,
                                             typename Elem<T>::acc (&out)[16]) {
    using A = typename Elem<T>::acc;
    if (vec && valid >= 16) {
        if constexpr (sizeof(T) == 4) {
            const float4* p = reinterpret_cast<const float4*>(src);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                float4 x = __ldg(p + v);
                out[4 * v + 0] = x.x; out[4 * v + 1] = x.y; out[4 * v + 2] = x.z; out[4 * v + 3] = x.w;
            }
            return;
        } else if constexpr (sizeof(T) == 2) {
            const uint4* p = reinterpret_cast<const uint4*>(src);
#pragma unroll
            for (int v = 0; v < 2; ++v) {
                uint4 x = __ldg(p + v);
                const T* h = reinterpret_cast<const T*>(&x);
#pragma unroll
                for (int e = 0; e < 8; ++e) out[8 * v + e] = Elem<T>::load(h[e]);
            }
            return;
        }
    }
#pragma unroll
    for (int e = 0; e < 16; ++e) out[e] = (e < valid) ? Elem<T>::load(src[e]) : A(0);
}

template <typename A>
__device__ __forceinline__ A absdiff_acc(A acc, A q, A k) {
    if constexpr (sizeof(A) == 4) {
        return add_abs_ftz(acc, sub_ftz(q, k));
    } else {
        A d = q - k;
        return acc + fabs(d);
    }
}

// acc[r][j] += |q[r][c] - k[j][c]| for the DR channels of one register
// chunk, in channel order.  FULL unrolls the whole chunk; otherwise `valid`
// channels (ragged last chunk) are taken at run time.
template <typename A, int TM, int MC, int DR, bool FULL>
__device__ __forceinline__ void accum_chunk(A (&acc)[TM][MC], const A (&qr)[TM][DR], const A* kbase, int DP,
                                            int valid = DR) {
#pragma unroll
    for (int j = 0; j < MC; ++j) {
        const A* kr = kbase + j * DP;
#pragma unroll
        for (int c4 = 0; c4 < DR / 4; ++c4) {
            if (!FULL && c4 * 4 >= valid) break;
            A kv[4];
            if constexpr (sizeof(A) == 4) {
                float4 t = *reinterpret_cast<const float4*>(kr + 4 * c4);
                kv[0] = t.x; kv[1] = t.y; kv[2] = t.z; kv[3] = t.w;
            } else {
#pragma unroll
                for (int e = 0; e < 4; ++e) kv[e] = kr[4 * c4 + e];
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                if (FULL || 4 * c4 + e < valid) {
#pragma unroll
                    for (int r = 0; r < TM; ++r) acc[r][j] = absdiff_acc<A>(acc[r][j], qr[r][4 * c4 + e], kv[e]);
                }
            }
        }
    }
}

// Forward epilogue: S itself, or exp(escale * S) for the Laplacian kernel
// matrix (the attention block's exp(-S/sigma)); the exponential is CUDA's
// expf / exp on the accumulation type.
template <typename A>
__device__ __forceinline__ A fwd_epilogue(A acc, A escale, bool do_exp) {
    if (!do_exp) return acc;
    if constexpr (sizeof(A) == 4) return expf(escale * acc);
    else return exp(escale * acc);
}

// One CTA = kThreads*TM query rows of one (b,h); thread t owns rows
// base + t + kThreads*r and keeps DR channels of each in registers.  When
// d <= DR the rows are loaded once and zero padded to DR (padded channels add
// |0 - 0| = +0, which leaves every sum unchanged); otherwise the channels are
// walked in DR-wide chunks.  ks holds KT transposed to [m][DP] in the
// accumulation type (DP = max(DR, d rounded up to 16), zero padded).
// Landmark windows: CTA (x, y) computes landmarks [y*mwin, y*mwin + m) of
// its rows (m = min(mwin, mfull - y*mwin)); mfull is the row stride of S
// and K^T.  More, smaller CTAs fill the last wave of a small grid better.
template <typename T, int TM, int MC, int DR>
__global__ void __launch_bounds__(kThreads)
lsub_fwd_kernel(const T* __restrict__ q, const T* __restrict__ kT, T* __restrict__ s,
                int n, int mfull, int mwin, int d, int tiles_per_bh, bool vec, int gw,
                typename Elem<T>::acc escale, bool do_exp) {
    using A = typename Elem<T>::acc;
    const int j_off = (int)blockIdx.y * mwin;
    const int m = min(mwin, mfull - j_off);
    extern __shared__ __align__(16) unsigned char smem_raw[];
    A* ks = reinterpret_cast<A*>(smem_raw);
    const int d16 = (d + 15) & ~15;
    const int DP = d16 > DR ? ((d + DR - 1) / DR) * DR : DR;
    const int MP = ((m + MC - 1) / MC) * MC;
    // Output tile [kThreads*TM][gw] in the storage type, after ks (16-byte
    // aligned), gw = m or a multiple of MC (landmark groups of gw columns
    // when the whole tile would not fit); written row-wise by the lanes and
    // copied out with 16-byte stores: one contiguous run of S when gw = m,
    // row segments of gw columns otherwise.  gw = 0: direct stores.
    T* so = reinterpret_cast<T*>(smem_raw + (((size_t)MP * DP * sizeof(A) + 15) & ~(size_t)15));
    const bool single = d <= DR;

    const int bh = blockIdx.x / tiles_per_bh;
    const int tile = blockIdx.x - bh * tiles_per_bh;
    const T* Kb = kT + (int64_t)bh * d * mfull + j_off;

    // Stage KT[bh] (d x m, row-major) transposed into ks[j][c].
    for (int e = threadIdx.x; e < MP * DP; e += kThreads) {
        int j = e / DP, c = e - j * DP;
        ks[e] = (j < m && c < d) ? Elem<T>::load(Kb[(int64_t)c * mfull + j]) : A(0);
    }
    __syncthreads();

    const int64_t row0 = (int64_t)tile * (kThreads * TM) + threadIdx.x;
    const T* Qb = q + (int64_t)bh * n * d;
    T* Sb = s + (int64_t)bh * n * mfull + j_off;

    A qr[TM][DR];
    auto load_q = [&](int dc) {
#pragma unroll
        for (int r = 0; r < TM; ++r) {
            int64_t row = row0 + (int64_t)kThreads * r;
            if constexpr (DR == 8) {
                const int valid = d - dc;
                if (row < n && valid >= 8 && vec && sizeof(T) == 4) {
                    const float4* p = reinterpret_cast<const float4*>(Qb + row * d + dc);
                    float4 x0 = __ldg(p), x1 = __ldg(p + 1);
                    qr[r][0] = x0.x; qr[r][1] = x0.y; qr[r][2] = x0.z; qr[r][3] = x0.w;
                    qr[r][4] = x1.x; qr[r][5] = x1.y; qr[r][6] = x1.z; qr[r][7] = x1.w;
                } else {
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        qr[r][e] = (row < n && e < valid) ? Elem<T>::load(Qb[row * d + dc + e]) : A(0);
                }
            } else {
#pragma unroll
                for (int x = 0; x < DR / 16; ++x) {
                    A(&dst)[16] = *reinterpret_cast<A(*)[16]>(&qr[r][16 * x]);
                    const int valid = d - dc - 16 * x;
                    if (row < n && valid > 0) {
                        load_chunk16<T>(Qb + row * d + dc + 16 * x, valid, vec, dst);
                    } else {
#pragma unroll
                        for (int e = 0; e < 16; ++e) dst[e] = A(0);
                    }
                }
            }
        }
    };
    if (single) load_q(0);

    int g0 = 0;  // first landmark of the staged group
    const int64_t trow = (int64_t)tile * (kThreads * TM);
    const int64_t rows = (n - trow) < (int64_t)(kThreads * TM) ? (n - trow) : (int64_t)(kThreads * TM);
    for (int mc = 0; mc < m; mc += MC) {
        A acc[TM][MC];
#pragma unroll
        for (int r = 0; r < TM; ++r)
#pragma unroll
            for (int j = 0; j < MC; ++j) acc[r][j] = A(0);

        if (single) {
            accum_chunk<A, TM, MC, DR, true>(acc, qr, ks + mc * DP, DP);
        } else {
            for (int dc = 0; dc < d; dc += DR) {
                load_q(dc);
                if (d - dc >= DR) accum_chunk<A, TM, MC, DR, true>(acc, qr, ks + mc * DP + dc, DP);
                else accum_chunk<A, TM, MC, DR, false>(acc, qr, ks + mc * DP + dc, DP, d - dc);
            }
        }
#pragma unroll
        for (int r = 0; r < TM; ++r) {
            if (gw) {
                T* out = so + (threadIdx.x + kThreads * r) * gw + (mc - g0);
#pragma unroll
                for (int j = 0; j < MC; ++j)
                    if (mc + j < m) out[j] = Elem<T>::store(fwd_epilogue(acc[r][j], escale, do_exp));
                continue;
            }
            int64_t row = row0 + (int64_t)kThreads * r;
            if (row >= n) continue;
            T* out = Sb + row * mfull + mc;
#pragma unroll
            for (int j = 0; j < MC; ++j)
                if (mc + j < m) out[j] = Elem<T>::store(fwd_epilogue(acc[r][j], escale, do_exp));
        }
        if (gw && (mc + MC >= g0 + gw || mc + MC >= m)) {
            __syncthreads();
            const int w = (m - g0) < gw ? (m - g0) : gw;
            constexpr int V = 16 / sizeof(T);
            if (w == m && m == mfull) {
                // the tile's rows are one contiguous run of S
                const int64_t cnt = rows * m;
                T* dst = Sb + trow * m;
                int64_t head = 0;
                if ((reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
                    const int64_t nv = cnt / V;
                    const uint4* src4 = reinterpret_cast<const uint4*>(so);
                    uint4* dst4 = reinterpret_cast<uint4*>(dst);
                    for (int64_t e = threadIdx.x; e < nv; e += kThreads) dst4[e] = src4[e];
                    head = nv * V;
                }
                for (int64_t e = head + threadIdx.x; e < cnt; e += kThreads) dst[e] = so[e];
            } else {
                T* dst = Sb + trow * mfull + g0;
                const bool v16 = (w % V == 0) && (mfull % V == 0) && (gw % V == 0) &&
                                 (reinterpret_cast<uintptr_t>(dst) & 15) == 0;
                if (v16) {
                    const int U = w / V;
                    for (int64_t e = threadIdx.x; e < rows * U; e += kThreads) {
                        const int64_t r = e / U;
                        const int u = (int)(e - r * U);
                        *reinterpret_cast<uint4*>(dst + r * mfull + u * V) =
                            *reinterpret_cast<const uint4*>(so + r * gw + u * V);
                    }
                } else {
                    for (int64_t e = threadIdx.x; e < rows * w; e += kThreads) {
                        const int64_t r = e / w;
                        const int cc = (int)(e - r * w);
                        dst[r * mfull + cc] = so[r * gw + cc];
                    }
                }
            }
            __syncthreads();
            g0 += gw;
        }
    }
}

// Landmark chunk per thread: the MC in 4..8 that pads m the least.
int pick_mc(int64_t m) {
    int best = 8;
    int64_t best_pad = ((m + 7) / 8) * 8;
    for (int c = 7; c >= 4; --c) {
        int64_t pad = ((m + c - 1) / c) * c;
        if (pad < best_pad) { best = c; best_pad = pad; }
    }
    return best;
}

template <typename T, int TM, int MC, int DR>
size_t fwd_smem(int64_t m, int64_t d) {
    using A = typename Elem<T>::acc;
    const int d16 = (int)((d + 15) & ~15);
    const int DP = d16 > DR ? (int)(((d + DR - 1) / DR) * DR) : DR;
    const int MP = (int)(((m + MC - 1) / MC) * MC);
    return (size_t)MP * DP * sizeof(A);
}

// Landmark columns of the staged output tile: all m when the tile fits in
// kStageMax bytes (more would cost occupancy), else the widest multiple of MC
// that does (landmark groups); 0 (direct stores) below 2*MC columns.
constexpr size_t kStageMax = 64 * 1024;
template <typename T, int TM, int MC>
int fwd_stage_width(int64_t m) {
    const size_t row_bytes = (size_t)kThreads * TM * sizeof(T);
    if ((size_t)m * row_bytes <= kStageMax) return (int)m;
    const int64_t w = (int64_t)(kStageMax / row_bytes) / MC * MC;
    return w >= 2 * MC ? (int)w : 0;
}
template <typename T, int TM, int MC>
size_t fwd_stage_bytes(int64_t m) {
    return (size_t)kThreads * TM * fwd_stage_width<T, TM, MC>(m) * sizeof(T);
}

template <typename T, int TM, int MC, int DR>
size_t fwd_smem_total(int64_t m, int64_t d) {
    size_t st = fwd_stage_bytes<T, TM, MC>(m);
    size_t ks = fwd_smem<T, TM, MC, DR>(m, d);
    return st ? ((ks + 15) & ~(size_t)15) + st : ks;
}

template <typename T, int TM, int MC, int DR>
int launch_fwd_mc(const T* q, const T* kT, T* s, int64_t bh, int64_t n, int64_t m, int64_t d,
                  cudaStream_t st, double escale, bool do_exp) {
    auto kern = lsub_fwd_kernel<T, TM, MC, DR>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, max_optin_smem());
    const int tiles = (int)((n + kThreads * TM - 1) / (kThreads * TM));
    // Shared memory and staged-output width for landmark windows of mw columns.
    auto plan = [&](int64_t mw, size_t& smem, int& gw) {
        smem = fwd_smem_total<T, TM, MC, DR>(mw, d);
        gw = fwd_stage_width<T, TM, MC>(mw);
        // Narrower landmark groups when that lets two CTAs share an SM (the
        // staged K^T and the output tile of one CTA otherwise fill more than
        // half of its shared memory, leaving 8 warps per SM).
        const size_t half_sm = (size_t)max_optin_smem() / 2 - 1024;
        const size_t ksb = (fwd_smem<T, TM, MC, DR>(mw, d) + 15) & ~(size_t)15;
        const size_t row_bytes = (size_t)kThreads * TM * sizeof(T);
        if (gw > 0 && smem > half_sm && ksb + 2 * MC * row_bytes <= half_sm) {
            gw = (int)(((half_sm - ksb) / row_bytes) / MC * MC);
            smem = ksb + (size_t)gw * row_bytes;
        }
        if (gw == 0 || smem > (size_t)max_optin_smem()) {
            gw = 0;
            smem = fwd_smem<T, TM, MC, DR>(mw, d);
        }
    };
    // Landmark windows: 1, 2 or 4 (each a multiple of MC landmarks), chosen
    // by the estimated time waves x (landmarks per CTA + a query-row load
    // worth ~MC landmarks); ties keep fewer windows.
    int64_t mw = m;
    size_t smem = 0;
    int gw = 0;
    plan(m, smem, gw);
    double best = -1.0;
    for (int nw = 1; nw <= 4; nw *= 2) {
        // (one window is exactly m wide: the staged tile is then one contiguous run of S)
        const int64_t w = nw == 1 ? m : ((m + nw - 1) / nw + MC - 1) / MC * MC;
        if (nw > 1 && w < 4 * MC) break;
        const int64_t nwin = (m + w - 1) / w;
        size_t sm_w;
        int gw_w;
        plan(w, sm_w, gw_w);
        if (sm_w > (size_t)max_optin_smem()) continue;
        const int64_t slots = cta_slots(kern, sm_w);
        const int64_t blocks = bh * tiles * nwin;
        const double est = (double)((blocks + slots - 1) / slots) * (double)(w + MC);
        if (best < 0 || est < best * 0.97) { best = est; mw = w; smem = sm_w; gw = gw_w; }
    }
    if (smem > (size_t)max_optin_smem()) {
        set_error("LaplaceSubtraction forward: m*d = %lld*%lld needs %zu bytes of shared memory",
                  (long long)m, (long long)d, smem);
        return LF_ERR_UNSUPPORTED;
    }
    const int64_t nwin = (m + mw - 1) / mw;
    int64_t blocks = bh * tiles;
    if (blocks > 0x7fffffff || nwin > 65535) { set_error("too many blocks"); return LF_ERR_UNSUPPORTED; }
    bool vec = (d % 16 == 0) && aligned(q, 16);
    kern<<<dim3((unsigned)blocks, (unsigned)nwin), kThreads, smem, st>>>(q, kT, s, (int)n, (int)m, (int)mw, (int)d,
                                                                        tiles, vec, gw,
                                                                        (typename Elem<T>::acc)escale, do_exp);
    return check_launch("lsub_fwd_kernel");
}

// Two rows per thread amortise each landmark load over more terms; one row
// per thread halves the CTA's rows (twice the CTAs).  The choice compares
// the estimated times of the two grids.
template <typename T, int MC, int DR>
int launch_fwd_tm(const T* Q, const T* K, T* S, int64_t bh, int64_t n, int64_t m, int64_t d, cudaStream_t st,
                 double escale, bool do_exp) {
    if constexpr (DR <= 32) {
        const size_t smem1 = fwd_smem_total<T, 1, MC, DR>(m, d);
        const size_t smem2 = fwd_smem_total<T, 2, MC, DR>(m, d);
        if (smem1 <= (size_t)max_optin_smem() && smem2 <= (size_t)max_optin_smem()) {
            auto k1 = lsub_fwd_kernel<T, 1, MC, DR>;
            auto k2 = lsub_fwd_kernel<T, 2, MC, DR>;
            if (smem1 > 48 * 1024) cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem1);
            if (smem2 > 48 * 1024) cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem2);
            // Estimated time in one-row CTA times: waves x rows per thread
            // (a two-row CTA costs ~1.8 one-row CTAs: the landmark loads are
            // shared).  Small grids (under one wave) thus take one row.
            const int64_t s1 = cta_slots(k1, smem1), s2 = cta_slots(k2, smem2);
            const int64_t n1 = bh * ((n + kThreads - 1) / kThreads);
            const int64_t n2 = bh * ((n + 2 * kThreads - 1) / (2 * kThreads));
            const double t1 = (double)((n1 + s1 - 1) / s1);
            const double t2 = 1.8 * (double)((n2 + s2 - 1) / s2);
            if (t1 <= t2) return launch_fwd_mc<T, 1, MC, DR>(Q, K, S, bh, n, m, d, st, escale, do_exp);
        }
        return launch_fwd_mc<T, 2, MC, DR>(Q, K, S, bh, n, m, d, st, escale, do_exp);
    } else {
        return launch_fwd_mc<T, 1, MC, DR>(Q, K, S, bh, n, m, d, st, escale, do_exp);
    }
}

template <typename T, int DR>
int launch_fwd_dr(const T* Q, const T* K, T* S, int64_t bh, int64_t n, int64_t m, int64_t d, cudaStream_t st,
                 double escale, bool do_exp) {
    switch (pick_mc(m)) {
        case 4: return launch_fwd_tm<T, 4, DR>(Q, K, S, bh, n, m, d, st, escale, do_exp);
        case 5: return launch_fwd_tm<T, 5, DR>(Q, K, S, bh, n, m, d, st, escale, do_exp);
        case 6: return launch_fwd_tm<T, 6, DR>(Q, K, S, bh, n, m, d, st, escale, do_exp);
        case 7: return launch_fwd_tm<T, 7, DR>(Q, K, S, bh, n, m, d, st, escale, do_exp);
        default: return launch_fwd_tm<T, 8, DR>(Q, K, S, bh, n, m, d, st, escale, do_exp);
    }
}

// Register chunk: the whole row when d <= 64 (16 / 32 channels x 1-2 rows,
// or 64 channels x 1 row), 32-channel chunks beyond; fp64 uses 16 channels.
template <typename T>
int launch_fwd(const void* q, const void* kT, void* s, int64_t bh, int64_t n, int64_t m, int64_t d,
               cudaStream_t st, double escale = 0.0, bool do_exp = false) {
    const T* Q = static_cast<const T*>(q);
    const T* K = static_cast<const T*>(kT);
    T* S = static_cast<T*>(s);
    if constexpr (sizeof(T) == 8) {
        return launch_fwd_dr<T, 16>(Q, K, S, bh, n, m, d, st, escale, do_exp);
    } else {
        if (d <= 16) return launch_fwd_dr<T, 16>(Q, K, S, bh, n, m, d, st, escale, do_exp);
        if (d <= 32) {
            return launch_fwd_dr<T, 32>(Q, K, S, bh, n, m, d, st, escale, do_exp);
        }
        if (d <= 64) return launch_fwd_dr<T, 64>(Q, K, S, bh, n, m, d, st, escale, do_exp);
        return launch_fwd_dr<T, 32>(Q, K, S, bh, n, m, d, st, escale, do_exp);
    }
}

// ---------------------------------------------------------------------------
// Fused backward
// ---------------------------------------------------------------------------
template <typename A>
__device__ __forceinline__ A step_of(A q, A k) {
    if constexpr (sizeof(A) == 4) {
        return half_step_ftz(sub_ftz(q, k));
    } else {
        A d = q - k;
        return d > A(0) ? A(1) : (d < A(0) ? A(0) : A(0.5));
    }
}

// Four backward terms (landmarks j..j+3 of one channel) in fp32: for each,
// d = q - k, t = sat(d*2^125 + 1/2), dq += g*t, dk_j += g*t — exactly four
// FP32-pipe instructions per term, written out so that nothing else is
// scheduled into the hot loop.
template <bool DQ, bool DK>
__device__ __forceinline__ void bwd_quad(float q, float k0, float k1, float k2, float k3, const float (&g)[4],
                                         float& dq, float& a0, float& a1, float& a2, float& a3) {
    float t0, t1, t2, t3;
    asm("{\n\t.reg .f32 d0, d1, d2, d3;\n\t"
        "sub.rn.ftz.f32 d0, %4, %5;\n\t"
        "sub.rn.ftz.f32 d1, %4, %6;\n\t"
        "sub.rn.ftz.f32 d2, %4, %7;\n\t"
        "sub.rn.ftz.f32 d3, %4, %8;\n\t"
        "fma.rn.ftz.sat.f32 %0, d0, 0f7E000000, 0f3F000000;\n\t"
        "fma.rn.ftz.sat.f32 %1, d1, 0f7E000000, 0f3F000000;\n\t"
        "fma.rn.ftz.sat.f32 %2, d2, 0f7E000000, 0f3F000000;\n\t"
        "fma.rn.ftz.sat.f32 %3, d3, 0f7E000000, 0f3F000000;\n\t}"
        : "=f"(t0), "=f"(t1), "=f"(t2), "=f"(t3)
        : "f"(q), "f"(k0), "f"(k1), "f"(k2), "f"(k3));
    if (DQ) {
        dq = __fmaf_rn(g[0], t0, dq);
        dq = __fmaf_rn(g[1], t1, dq);
        dq = __fmaf_rn(g[2], t2, dq);
        dq = __fmaf_rn(g[3], t3, dq);
    }
    if (DK) {
        a0 = __fmaf_rn(g[0], t0, a0);
        a1 = __fmaf_rn(g[1], t1, a1);
        a2 = __fmaf_rn(g[2], t2, a2);
        a3 = __fmaf_rn(g[3], t3, a3);
    }
}

// The same four terms with both gradients, using the packed fp32x2 forms of
// sub and fma (sm_100): 2 sub.f32x2 + 4 fma.sat + 2+2 fma.f32x2 = 10 issued
// instructions instead of 16.  The FP32 pipe does the same work per term
// (a packed instruction occupies it twice as long), so this frees issue
// slots for the shared-memory loads and loop overhead, which otherwise
// compete with the arithmetic.  qq = {q, q}; dq accumulates in four
// partials (one per landmark of the quad).
__device__ __forceinline__ void bwd_quad_x2(unsigned long long qq, float k0, float k1, float k2, float k3,
                                            const float (&g)[4], float (&dq)[4],
                                            float& a0, float& a1, float& a2, float& a3) {
    asm("{\n\t.reg .b64 k01, k23, d01, d23, t01, t23, g01, g23, q01, q23, a01, a23;\n\t"
        ".reg .f32 d0, d1, d2, d3, t0, t1, t2, t3;\n\t"
        "mov.b64 k01, {%9, %10};\n\t"
        "mov.b64 k23, {%11, %12};\n\t"
        "sub.rn.ftz.f32x2 d01, %8, k01;\n\t"
        "sub.rn.ftz.f32x2 d23, %8, k23;\n\t"
        "mov.b64 {d0, d1}, d01;\n\t"
        "mov.b64 {d2, d3}, d23;\n\t"
        "fma.rn.ftz.sat.f32 t0, d0, 0f7E000000, 0f3F000000;\n\t"
        "fma.rn.ftz.sat.f32 t1, d1, 0f7E000000, 0f3F000000;\n\t"
        "fma.rn.ftz.sat.f32 t2, d2, 0f7E000000, 0f3F000000;\n\t"
        "fma.rn.ftz.sat.f32 t3, d3, 0f7E000000, 0f3F000000;\n\t"
        "mov.b64 t01, {t0, t1};\n\t"
        "mov.b64 t23, {t2, t3};\n\t"
        "mov.b64 g01, {%13, %14};\n\t"
        "mov.b64 g23, {%15, %16};\n\t"
        "mov.b64 q01, {%0, %1};\n\t"
        "mov.b64 q23, {%2, %3};\n\t"
        "mov.b64 a01, {%4, %5};\n\t"
        "mov.b64 a23, {%6, %7};\n\t"
        "fma.rn.f32x2 q01, g01, t01, q01;\n\t"
        "fma.rn.f32x2 q23, g23, t23, q23;\n\t"
        "fma.rn.f32x2 a01, g01, t01, a01;\n\t"
        "fma.rn.f32x2 a23, g23, t23, a23;\n\t"
        "mov.b64 {%0, %1}, q01;\n\t"
        "mov.b64 {%2, %3}, q23;\n\t"
        "mov.b64 {%4, %5}, a01;\n\t"
        "mov.b64 {%6, %7}, a23;\n\t}"
        : "+f"(dq[0]), "+f"(dq[1]), "+f"(dq[2]), "+f"(dq[3]), "+f"(a0), "+f"(a1), "+f"(a2), "+f"(a3)
        : "l"(qq), "f"(k0), "f"(k1), "f"(k2), "f"(k3), "f"(g[0]), "f"(g[1]), "f"(g[2]), "f"(g[3]));
}

constexpr int kRowChunk = 64;       // query rows staged per pass (at most)
constexpr int kMaxColChunks = 16;   // landmarks <= 512 = 16 x 32 lanes

struct BwdGeom {
    int n, m, d;
    int DBC;          // channel blocks (of 32 lanes) per CTA; grid.z covers the rest
    int MCN, RG;      // landmark chunks, row groups
    int MP;           // landmark stride of the staged gradient tile
    int KSTR;         // row stride of the per-CTA dKT accumulator (odd, conflict free)
    int rows_per_cta;
    int RC;           // query rows staged per pass (<= kRowChunk)
    // Balanced (flat) launch of the fast backward: the bh*U row chunks of
    // kRowChunk rows (U = chunks per (b,h)) are dealt out as contiguous runs
    // of P chunks per CTA.
    int64_t U, P, total;
    // Laplacian-kernel backward: when km is set, the upstream gradient is
    // dKmat and the kernels stage dS = kscale * km * dKmat (km = exp(kscale *
    // S), same layout as dS) as they load it.
    const void* km = nullptr;
    float kscale = 0.f;
    // Extra dQ destinations (peer GPUs' gather buffers, same element offsets),
    // stored by the wide kernel beside dq (lf_laplace_sub_bwd_peers).
    void* dqx[LF_MAX_PEERS] = {};
    int ndqx = 0;
};

// The optional dS factor of the Laplacian-kernel backward (see BwdGeom::km)
// and the extra dQ destinations of the wide kernel (see BwdGeom::dqx).
struct GFuse {
    const void* km = nullptr;
    float kscale = 0.f;
    void* const* dqx = nullptr;
    int ndqx = 0;
};

// Shapes the balanced wide backward runs (configuration-5 channels and
// landmarks); the others use the fast kernel or no workspace.
inline bool wide_flat_shape(int64_t m, int64_t d) { return d > 32 && d <= 64 && m > 128 && m <= 256; }

// dS value at index e of the (b,h) slice: g[e], or kscale * km[e] * g[e].
template <typename T>
__device__ __forceinline__ typename Elem<T>::acc grad_at(const T* __restrict__ gb, const T* __restrict__ kmb,
                                                         float kscale, int64_t e) {
    using A = typename Elem<T>::acc;
    A v = Elem<T>::load(gb[e]);
    if (kmb) v = (v * Elem<T>::load(kmb[e])) * (A)kscale;
    return v;
}

// grid = (cs, bh, channel groups), cluster = (cs, 1, 1).  CTA x of (b,h)
// handles query rows [x*rows_per_cta, (x+1)*rows_per_cta) for channels
// [z*32*DBC, (z+1)*32*DBC).  Warp w works on channel block w % DBC, landmark
// chunk (w / DBC) % MCN and row group w / (DBC*MCN).
//
// Per 64-row chunk the CTA stages 2*dS and Q in shared memory (coalesced row
// loads), with the row sums sum_j dS (warp shuffles) and the per-landmark
// column sums sum_i dS (shared atomics, accumulated over the CTA's rows).
template <typename T, int MB, bool DQ, bool DK, int MINB>
__global__ void __launch_bounds__(kThreads, MINB)
lsub_bwd_kernel(const T* __restrict__ g, const T* __restrict__ q, const T* __restrict__ kT,
                T* __restrict__ dq, T* __restrict__ dk, BwdGeom geo) {
    using A = typename Elem<T>::acc;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int n = geo.n, m = geo.m, d = geo.d;
    const int MP = geo.MP;
    const int RC = geo.RC;  // query rows staged per pass
    const int CW = geo.DBC * 32;  // channels per CTA
    // Shared memory carve-up (accumulation type):
    //   gs   [RC][MP]   2*dS of the staged rows (zero padded)
    //   qs   [RC][CW]   Q of the staged rows, this CTA's channels
    //   rsum [RC]       sum_j dS of each staged row
    //   dqb  [RC][CW]   dQ partials when MCN > 1
    //   csum [MP]              sum_i dS over the CTA's rows, per landmark
    //   dkb  [CW][KSTR]        dKT partials of this CTA
    //   cpart[8][MP]           per-warp partial column sums (each (warp, j)
    //                          is owned by one thread: no atomics)
    A* gs = reinterpret_cast<A*>(smem_raw);
    A* qs = gs + RC * MP;
    A* rsum = qs + RC * CW;
    A* dqb = rsum + RC;
    A* csum = dqb + (geo.MCN > 1 ? RC * CW : 0);
    A* dkb = csum + MP;
    A* cpart = dkb + (DK ? CW * geo.KSTR : 0);  // [8 warps][MP] column-sum partials

    cg::cluster_group cluster = cg::this_cluster();
    const int bh = blockIdx.y;
    const int split = blockIdx.x;
    const int c0 = blockIdx.z * CW;              // first channel of this CTA
    const int cw = min(CW, d - c0);              // channels of this CTA
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int groups = geo.DBC * geo.MCN;
    const int db = warp % geo.DBC;
    const int mcb = (warp / geo.DBC) % geo.MCN;
    const int rg = warp / groups;
    const bool warp_active = rg < geo.RG;
    const int cl = db * 32 + lane;               // channel within the CTA
    const int c = c0 + cl;
    const bool lane_active = warp_active && cl < cw;
    const int j0 = mcb * MB;

    const T* Gb = g + (int64_t)bh * n * m;
    const T* Qb = q + (int64_t)bh * n * d;
    const T* Kb = kT + (int64_t)bh * d * m;

    if (DK) {
        for (int e = threadIdx.x; e < CW * geo.KSTR; e += kThreads) dkb[e] = A(0);
        for (int e = threadIdx.x; e < MP; e += kThreads) csum[e] = A(0);
        for (int e = threadIdx.x; e < (kThreads / 32) * MP; e += kThreads) cpart[e] = A(0);
    }

    // Landmark values of this lane's channel and its dKT partials.
    A kreg[MB];
    A dka[MB];
#pragma unroll
    for (int jj = 0; jj < MB; ++jj) {
        int j = j0 + jj;
        kreg[jj] = (lane_active && j < m) ? Elem<T>::load(Kb[(int64_t)c * m + j]) : A(0);
        dka[jj] = A(0);
    }

    const int64_t r_begin = (int64_t)split * geo.rows_per_cta;
    const int64_t r_end = (r_begin + geo.rows_per_cta < (int64_t)n) ? r_begin + geo.rows_per_cta : (int64_t)n;

    for (int64_t rc = r_begin; rc < r_end; rc += RC) {
        const int rows = (int)((r_end - rc) < RC ? (r_end - rc) : RC);
        __syncthreads();  // previous chunk fully consumed
        // Stage the chunk: warp w takes rows w, w+8, ...; lanes walk the row.
        for (int i = warp; i < RC; i += kThreads / 32) {
            const bool row_ok = i < rows;
            const T* grow = Gb + (rc + i) * m;
            const T* kmrow = geo.km ? static_cast<const T*>(geo.km) + (grow - g) : nullptr;
            A rs = A(0);
#pragma unroll
            for (int u = 0; u < kMaxColChunks; ++u) {
                const int j = lane + 32 * u;
                if (j < MP) {
                    A v = (row_ok && j < m) ? grad_at<T>(grow, kmrow, geo.kscale, j) : A(0);
                    gs[i * MP + j] = v + v;
                    rs += v;
                    if (DK) cpart[warp * MP + j] += v;
                }
            }
            if (DQ) {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, o);
                if (lane == 0) rsum[i] = rs;
            }
            const T* qrow = Qb + (rc + i) * d + c0;
            for (int x = lane; x < CW; x += 32)
                qs[i * CW + x] = (row_ok && x < cw) ? Elem<T>::load(qrow[x]) : A(0);
            if (DQ && geo.MCN > 1)
                for (int x = lane; x < CW; x += 32) dqb[i * CW + x] = A(0);
        }
        __syncthreads();

        if (lane_active) {
#pragma unroll 1
            for (int i = rg; i < rows; i += geo.RG) {
                const A qv = qs[i * CW + cl];
                const A* grow = gs + i * MP + j0;
                A dqa = A(0);
#pragma unroll
                for (int j4 = 0; j4 < MB; j4 += 4) {
                    A gv[4];
                    if constexpr (sizeof(A) == 4) {
                        float4 t4 = *reinterpret_cast<const float4*>(grow + j4);
                        gv[0] = t4.x; gv[1] = t4.y; gv[2] = t4.z; gv[3] = t4.w;
                    } else {
#pragma unroll
                        for (int e = 0; e < 4; ++e) gv[e] = grow[j4 + e];
                    }
                    if constexpr (sizeof(A) == 4) {
                        bwd_quad<DQ, DK>(qv, kreg[j4], kreg[j4 + 1], kreg[j4 + 2], kreg[j4 + 3], gv, dqa,
                                         dka[j4], dka[j4 + 1], dka[j4 + 2], dka[j4 + 3]);
                    } else {
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const A t = step_of<A>(qv, kreg[j4 + e]);
                            if (DQ) dqa = fma_acc(gv[e], t, dqa);
                            if (DK) dka[j4 + e] = fma_acc(gv[e], t, dka[j4 + e]);
                        }
                    }
                }
                if (DQ) {
                    if (geo.MCN == 1) {
                        dq[((int64_t)bh * n + rc + i) * d + c] = Elem<T>::store(dqa - rsum[i]);
                    } else {
                        atomicAdd(&dqb[i * CW + cl], mcb == 0 ? dqa - rsum[i] : dqa);
                    }
                }
            }
        }
        if (DQ && geo.MCN > 1) {
            __syncthreads();
            for (int i = warp; i < rows; i += kThreads / 32)
                for (int x = lane; x < cw; x += 32)
                    dq[((int64_t)bh * n + rc + i) * d + c0 + x] = Elem<T>::store(dqb[i * CW + x]);
        }
    }

    if (!DK) return;

    __syncthreads();
    for (int j = threadIdx.x; j < m; j += kThreads) {
        A sacc = A(0);
        for (int w = 0; w < kThreads / 32; ++w) sacc += cpart[w * MP + j];
        csum[j] = sacc;
    }
    // dKT[c][j] = csum[j] - sum_i 2g*t, first within the CTA ...
    if (lane_active) {
#pragma unroll
        for (int jj = 0; jj < MB; ++jj) {
            int j = j0 + jj;
            if (j < m) atomicAdd(&dkb[cl * geo.KSTR + j], -dka[jj]);
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < cw * m; e += kThreads) {
        int cc = e / m, j = e - cc * m;
        dkb[cc * geo.KSTR + j] += csum[j];
    }
    // ... then across the cluster through distributed shared memory.
    cluster.sync();
    const int cs = (int)cluster.num_blocks();
    const int rank = (int)cluster.block_rank();
    const int total = cw * m;
    const int per = (total + cs - 1) / cs;
    const int e0 = rank * per, e1 = min(total, e0 + per);
    T* dkout = dk + (int64_t)bh * d * m + (int64_t)c0 * m;
    for (int e = e0 + threadIdx.x; e < e1; e += kThreads) {
        int cc = e / m, j = e - cc * m;
        A sacc = A(0);
        for (int r = 0; r < cs; ++r) {
            const A* peer = cluster.map_shared_rank(dkb, r);
            sacc += peer[cc * geo.KSTR + j];
        }
        dkout[e] = Elem<T>::store(sacc);
    }
    cluster.sync();  // keep this CTA's shared memory alive until peers are done
}

// Fast path of the fused backward for d <= 32 and m <= 64 (one channel
// block, one landmark chunk per warp): the pyramid-ViT shapes.  Staging maps
// four threads to each of the 64 rows of a chunk (thread (r, q) owns the
// landmark quarter q and channel octet q of row r), so row sums are two
// shuffles, column sums stay in registers for the whole CTA, and the next
// chunk's dS and Q are loaded into registers while the current one is being
// consumed.  Same arithmetic and cluster reduction as lsub_bwd_kernel.
//
// FLAT (both gradients only): no cluster; CTA i takes row chunks
// [i*P, (i+1)*P) of the flattened (b,h, chunk) order, which may cross (b,h)
// boundaries.  A (b,h) whose chunks all lie in one CTA gets its dKT written
// directly; the partial dKT of a (b,h) shared by several CTAs goes to
// workspace slot 2i (the CTA's first segment) or 2i+1 (its last), and
// lsub_bwd_dk_finalize adds the slots.  Every CTA-slot of the machine works
// (a per-(b,h) cluster leaves SMs idle when bh*cs is not a multiple of them).
//
// KM: the gradient is dKmat and the staging forms dS = kscale * Kmat * dKmat
// (BwdGeom::km); a separate instantiation, so the plain backward carries no
// trace of it (a runtime test in the staging loads cost the configuration-2
// backward 40 % of its speed).
template <typename T, int MB, bool DQ, bool DK, bool FLAT, bool KM>
__global__ void __launch_bounds__(kThreads, 1)
lsub_bwd_fast_kernel(const T* __restrict__ g, const T* __restrict__ q, const T* __restrict__ kT,
                     T* __restrict__ dq, T* __restrict__ dk, BwdGeom geo, float* __restrict__ ws) {
    using A = typename Elem<T>::acc;
    constexpr int RC = kRowChunk;   // 64 rows per chunk
    constexpr int CPT = MB / 4;     // landmarks per staging thread
    constexpr int CW = 32;          // channels (one block)
    constexpr int MP = MB;          // staged row stride
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int n = geo.n, m = geo.m, d = geo.d;
    A* gs = reinterpret_cast<A*>(smem_raw);  // [RC][MP]  dS (not doubled)
    A* qs = gs + RC * MP;                      // [RC][CW]
    A* rsum = qs + RC * CW;                    // [RC]
    A* csum = rsum + RC;                       // [MP]
    A* dkb = csum + MP;                        // [CW][KSTR]
    A* cpart = dkb + CW * geo.KSTR;            // [8][MP]
    A* dpart = cpart + (kThreads / 32) * MP;   // [8][CW][KSTR] per-warp dKT partials

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = lane;                 // this lane's channel
    const bool lane_active = c < d;
    const int rg = warp;                // row group (8 warps)
    const int sr = tid >> 2, sq = tid & 3;

    int64_t u = FLAT ? (int64_t)blockIdx.x * geo.P : 0;
    const int64_t u_end = FLAT ? ((u + geo.P < geo.total) ? u + geo.P : geo.total) : 1;
    for (int seg = 0; u < u_end; ++seg) {
    int bh;
    int64_t r_begin, r_end, u_next;
    if constexpr (FLAT) {
        bh = (int)(u / geo.U);
        const int64_t ub = (int64_t)bh * geo.U;
        u_next = (ub + geo.U < u_end) ? ub + geo.U : u_end;
        r_begin = (u - ub) * kRowChunk;
        r_end = (u_next - ub) * kRowChunk;
        if (r_end > n) r_end = n;
    } else {
        bh = blockIdx.y;
        r_begin = (int64_t)blockIdx.x * geo.rows_per_cta;
        r_end = (r_begin + geo.rows_per_cta < (int64_t)n) ? r_begin + geo.rows_per_cta : (int64_t)n;
        u_next = 1;
    }
    const T* Gb = g + (int64_t)bh * n * m;
    const T* Qb = q + (int64_t)bh * n * d;
    const T* Kb = kT + (int64_t)bh * d * m;

    A kreg[MB];
    A dka[MB];
#pragma unroll
    for (int jj = 0; jj < MB; ++jj) {
        kreg[jj] = (lane_active && jj < m) ? Elem<T>::load(Kb[(int64_t)c * m + jj]) : A(0);
        dka[jj] = A(0);
    }
    A colp[CPT];
#pragma unroll
    for (int k = 0; k < CPT; ++k) colp[k] = A(0);

    A pg[CPT], pq[8];
    const bool qvec = (d == 32) && ((reinterpret_cast<uintptr_t>(q) & 15) == 0);
    auto load_chunk = [&](int64_t rc) {
        const int64_t row = rc + sr;
        const bool ok = row < r_end;
        const T* grow = Gb + row * m + sq * CPT;
        const T* kmrow = KM ? static_cast<const T*>(geo.km) + (grow - g) : nullptr;
#pragma unroll
        for (int k = 0; k < CPT; ++k) {
            if constexpr (KM) pg[k] = (ok && sq * CPT + k < m) ? grad_at<T>(grow, kmrow, geo.kscale, k) : A(0);
            else pg[k] = (ok && sq * CPT + k < m) ? Elem<T>::load(grow[k]) : A(0);
        }
        const T* qrow = Qb + row * d + sq * 8;
        if (qvec && ok) {  // d == 32, 16-byte aligned rows: the eight values in one or two 16-byte loads
            if constexpr (sizeof(T) == 4) {
                const float4 a0 = __ldg(reinterpret_cast<const float4*>(qrow));
                const float4 a1 = __ldg(reinterpret_cast<const float4*>(qrow) + 1);
                pq[0] = a0.x; pq[1] = a0.y; pq[2] = a0.z; pq[3] = a0.w;
                pq[4] = a1.x; pq[5] = a1.y; pq[6] = a1.z; pq[7] = a1.w;
            } else {
                const uint4 u = __ldg(reinterpret_cast<const uint4*>(qrow));
                const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
                for (int k = 0; k < 8; ++k) pq[k] = Elem<T>::load(h[k]);
            }
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) pq[k] = (ok && sq * 8 + k < d) ? Elem<T>::load(qrow[k]) : A(0);
        }
    };
    if (r_begin < r_end) load_chunk(r_begin);

    for (int64_t rc = r_begin; rc < r_end; rc += RC) {
        const int rows = (int)((r_end - rc) < RC ? (r_end - rc) : RC);
        __syncthreads();  // previous chunk fully consumed
        {
            A rs = A(0);
#pragma unroll
            for (int k = 0; k < CPT; ++k) {
                gs[sr * MP + sq * CPT + k] = pg[k];
                rs += pg[k];
                if (DK) colp[k] += pg[k];
            }
            rs += __shfl_xor_sync(0xffffffffu, rs, 1);
            rs += __shfl_xor_sync(0xffffffffu, rs, 2);
            if (sq == 0) rsum[sr] = rs;
#pragma unroll
            for (int k = 0; k < 8; ++k) qs[sr * CW + sq * 8 + k] = pq[k];
        }
        __syncthreads();
        if (rc + RC < r_end) load_chunk(rc + RC);  // in flight during the compute below

        if (lane_active) {
#pragma unroll 1
            for (int i = rg; i < rows; i += kThreads / 32) {
                const A qv = qs[i * CW + c];
                const A* grow = gs + i * MP;
                A dqa = A(0);
                [[maybe_unused]] float dq4[4] = {0.f, 0.f, 0.f, 0.f};
                [[maybe_unused]] unsigned long long qq = 0;
                if constexpr (sizeof(A) == 4 && DQ && DK) asm("mov.b64 %0, {%1, %1};" : "=l"(qq) : "f"(qv));
#pragma unroll
                for (int j4 = 0; j4 < MB; j4 += 4) {
                    A gv[4];
                    if constexpr (sizeof(A) == 4 && DQ && DK) {
                        float4 t4 = *reinterpret_cast<const float4*>(grow + j4);
                        gv[0] = t4.x; gv[1] = t4.y; gv[2] = t4.z; gv[3] = t4.w;
                        bwd_quad_x2(qq, kreg[j4], kreg[j4 + 1], kreg[j4 + 2], kreg[j4 + 3], gv, dq4,
                                    dka[j4], dka[j4 + 1], dka[j4 + 2], dka[j4 + 3]);
                    } else if constexpr (sizeof(A) == 4) {
                        float4 t4 = *reinterpret_cast<const float4*>(grow + j4);
                        gv[0] = t4.x; gv[1] = t4.y; gv[2] = t4.z; gv[3] = t4.w;
                        bwd_quad<DQ, DK>(qv, kreg[j4], kreg[j4 + 1], kreg[j4 + 2], kreg[j4 + 3], gv, dqa,
                                         dka[j4], dka[j4 + 1], dka[j4 + 2], dka[j4 + 3]);
                    } else {
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            gv[e] = grow[j4 + e];
                            const A t = step_of<A>(qv, kreg[j4 + e]);
                            if (DQ) dqa = fma_acc(gv[e], t, dqa);
                            if (DK) dka[j4 + e] = fma_acc(gv[e], t, dka[j4 + e]);
                        }
                    }
                }
                if constexpr (sizeof(A) == 4 && DQ && DK) dqa = (dq4[0] + dq4[1]) + (dq4[2] + dq4[3]);
                // sum_j g*t was accumulated with g (not 2g): dQ = 2*acc - sum_j g
                if (DQ) dq[((int64_t)bh * n + rc + i) * d + c] = Elem<T>::store(A(2) * dqa - rsum[i]);
            }
        }
    }

    if (!DK) { u = u_next; continue; }

    // Column sums: reduce colp over the 8 rows of the warp that share a
    // quarter (lanes 4 apart), then across warps through shared memory.
#pragma unroll
    for (int k = 0; k < CPT; ++k) {
        A v = colp[k];
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 16);
        if (lane < 4) cpart[warp * MP + sq * CPT + k] = v;
    }
    // Per-warp partials of -2 * sum_i g*t, combined in a fixed order so that
    // results are bitwise reproducible.
    if (lane_active) {
#pragma unroll
        for (int jj = 0; jj < MB; ++jj)
            if (jj < m) dpart[(warp * CW + c) * geo.KSTR + jj] = A(-2) * dka[jj];
    }
    __syncthreads();
    for (int j = tid; j < m; j += kThreads) {
        A sacc = A(0);
        for (int w = 0; w < kThreads / 32; ++w) sacc += cpart[w * MP + j];
        csum[j] = sacc;
    }
    __syncthreads();
    for (int e = tid; e < d * m; e += kThreads) {
        int cc = e / m, j = e - cc * m;
        A sacc = csum[j];
        for (int w = 0; w < kThreads / 32; ++w) sacc += dpart[(w * CW + cc) * geo.KSTR + j];
        if constexpr (FLAT) {
            // Whole (b,h) in this CTA: final value; else a workspace slot.
            const bool whole = (u == (int64_t)bh * geo.U) && (u_next == (int64_t)bh * geo.U + geo.U);
            if (whole) dk[(int64_t)bh * d * m + e] = Elem<T>::store(sacc);
            else ws[((int64_t)2 * blockIdx.x + (seg == 0 ? 0 : 1)) * d * m + e] = (float)sacc;
        } else {
            dkb[cc * geo.KSTR + j] = sacc;
        }
    }
    if constexpr (FLAT) {
        __syncthreads();  // cpart/dpart/csum are reused by the next segment
        u = u_next;
        continue;
    } else {
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    const int cs = (int)cluster.num_blocks();
    const int rank = (int)cluster.block_rank();
    const int total = d * m;
    const int per = (total + cs - 1) / cs;
    const int e0 = rank * per, e1 = min(total, e0 + per);
    T* dkout = dk + (int64_t)bh * d * m;
    for (int e = e0 + tid; e < e1; e += kThreads) {
        int cc = e / m, j = e - cc * m;
        A sacc = A(0);
        for (int r = 0; r < cs; ++r) {
            const A* peer = cluster.map_shared_rank(dkb, r);
            sacc += peer[cc * geo.KSTR + j];
        }
        dkout[e] = Elem<T>::store(sacc);
    }
    cluster.sync();
    u = u_next;
    }
    }  // segments
}

// dKT of every (b,h) that the flat backward split over several CTAs: the
// sum of their workspace slots in CTA order (bitwise reproducible).  grid =
// (bh, element blocks): one element per thread; the slot loop keeps four
// independent partial sums (slots c0+4t+r go to partial r) that are combined
// in a fixed order, so the loads of a long slot list overlap.
template <typename T>
__global__ void __launch_bounds__(kThreads)
lsub_bwd_dk_finalize(const float* __restrict__ ws, T* __restrict__ dk, int d, int m, int64_t U, int64_t P) {
    const int64_t b = blockIdx.x;
    const int64_t first = b * U, last = b * U + U - 1;
    const int64_t c0 = first / P, c1 = last / P;
    if (c0 == c1) return;
    const int64_t dm = (int64_t)d * m;
    const int64_t e = (int64_t)blockIdx.y * kThreads + threadIdx.x;
    if (e >= dm) return;
    auto slot_val = [&](int64_t c) {
        const int64_t slot = 2 * c + (c * P >= first ? 0 : 1);
        return ws[slot * dm + e];
    };
    float p0 = 0.f, p1 = 0.f, p2 = 0.f, p3 = 0.f;
    int64_t c = c0;
    for (; c + 3 <= c1; c += 4) {
        p0 += slot_val(c);
        p1 += slot_val(c + 1);
        p2 += slot_val(c + 2);
        p3 += slot_val(c + 3);
    }
    if (c <= c1) p0 += slot_val(c);
    if (c + 1 <= c1) p1 += slot_val(c + 1);
    if (c + 2 <= c1) p2 += slot_val(c + 2);
    dk[b * dm + e] = Elem<T>::store((p0 + p1) + (p2 + p3));
}

template <typename T, int MB, bool DQ, bool DK>
int launch_bwd_fast(const T* g, const T* q, const T* kT, T* dq, T* dk, int64_t bh, int64_t n, int64_t m,
                    int64_t d, cudaStream_t st, GFuse fz = {}) {
    using A = typename Elem<T>::acc;
    BwdGeom geo;
    geo.n = (int)n; geo.m = (int)m; geo.d = (int)d;
    geo.km = fz.km; geo.kscale = fz.kscale;
    geo.DBC = 1; geo.MCN = 1; geo.RG = kThreads / 32; geo.MP = MB; geo.RC = kRowChunk;
    geo.KSTR = (int)(m | 1);
    size_t smem = sizeof(A) * ((size_t)kRowChunk * MB + (size_t)kRowChunk * 32 + kRowChunk + MB +
                               (size_t)32 * geo.KSTR + (size_t)(kThreads / 32) * MB +
                               (DK ? (size_t)(kThreads / 32) * 32 * geo.KSTR : 0));
    auto kern = fz.km ? lsub_bwd_fast_kernel<T, MB, DQ, DK, false, true> : lsub_bwd_fast_kernel<T, MB, DQ, DK, false, false>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const int64_t slots = cta_slots(kern, smem);
    const int64_t max_by_rows = (n + kRowChunk - 1) / kRowChunk;
    int64_t cs = 1;
    double best = -1.0;
    for (int64_t c = 1; c <= 8 && c <= (max_by_rows < 1 ? 1 : max_by_rows); ++c) {
        double eff = wave_efficiency(bh * c, slots);
        if (eff > best + 1e-9) { best = eff; cs = c; }
    }
    int64_t rpc = (n + cs - 1) / cs;
    rpc = ((rpc + kRowChunk - 1) / kRowChunk) * kRowChunk;
    geo.rows_per_cta = (int)rpc;
    if (bh > 65535) { set_error("b*h = %lld exceeds 65535", (long long)bh); return LF_ERR_UNSUPPORTED; }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)cs, (unsigned)bh, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t err = cudaLaunchKernelEx(&cfg, kern, g, q, kT, dq, dk, geo, (float*)nullptr);
    if (err != cudaSuccess) {
        set_error("lsub_bwd_fast_kernel launch: %s", cudaGetErrorString(err));
        return LF_ERR_CUDA;
    }
    return check_launch("lsub_bwd_fast_kernel");
}

// Balanced launch of the fast backward (both gradients).  With ws == nullptr
// only computes the workspace bytes into *need (0: this shape does not take
// the flat path).  Returns LF_OK, or an error when ws is given but smaller
// than needed.
template <typename T, int MB>
int launch_bwd_flat(const T* g, const T* q, const T* kT, T* dq, T* dk, int64_t bh, int64_t n, int64_t m,
                    int64_t d, float* ws, size_t ws_bytes, size_t* need, cudaStream_t st, GFuse fz = {}) {
    using A = typename Elem<T>::acc;
    BwdGeom geo;
    geo.n = (int)n; geo.m = (int)m; geo.d = (int)d;
    geo.km = fz.km; geo.kscale = fz.kscale;
    geo.DBC = 1; geo.MCN = 1; geo.RG = kThreads / 32; geo.MP = MB; geo.RC = kRowChunk;
    geo.KSTR = (int)(m | 1);
    geo.rows_per_cta = 0;
    size_t smem = sizeof(A) * ((size_t)kRowChunk * MB + (size_t)kRowChunk * 32 + kRowChunk + MB +
                               (size_t)32 * geo.KSTR + (size_t)(kThreads / 32) * MB +
                               (size_t)(kThreads / 32) * 32 * geo.KSTR);
    auto kern = fz.km ? lsub_bwd_fast_kernel<T, MB, true, true, true, true> : lsub_bwd_fast_kernel<T, MB, true, true, true, false>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const int64_t slots = cta_slots(kern, smem);
    geo.U = (n + kRowChunk - 1) / kRowChunk;
    geo.total = bh * geo.U;
    geo.P = (geo.total + slots - 1) / slots;
    const int64_t grid = (geo.total + geo.P - 1) / geo.P;
    const size_t bytes = (size_t)2 * grid * d * m * sizeof(float);
    if (need) *need = bytes;
    if (!ws) return LF_OK;
    if (ws_bytes < bytes) {
        set_error("LaplaceSubtraction backward: workspace of %zu bytes, %zu needed", ws_bytes, bytes);
        return LF_ERR_INVALID;
    }
    kern<<<(unsigned)grid, kThreads, smem, st>>>(g, q, kT, dq, dk, geo, ws);
    int rc = check_launch("lsub_bwd_fast_kernel");
    if (rc) return rc;
    if (bh > 0x7fffffff) { set_error("b*h too large"); return LF_ERR_UNSUPPORTED; }
    const unsigned eblocks = (unsigned)((d * m + kThreads - 1) / kThreads);
    lsub_bwd_dk_finalize<T><<<dim3((unsigned)bh, eblocks, 1), kThreads, 0, st>>>(ws, dk, (int)d, (int)m, geo.U, geo.P);
    return check_launch("lsub_bwd_dk_finalize");
}

template <typename T, int DBT, int MCNT, int MB, int NT>
int launch_bwd_wide_flat(const T* g, const T* q, const T* kT, T* dq, T* dk, int64_t bh, int64_t n, int64_t m,
                         int64_t d, float* ws, size_t ws_bytes, size_t* need, cudaStream_t st, GFuse fz = {});

template <typename T>
int launch_bwd_flat_t(const void* g, const void* q, const void* kT, void* dq, void* dk, int64_t bh, int64_t n,
                      int64_t m, int64_t d, void* ws, size_t ws_bytes, size_t* need, cudaStream_t st,
                      GFuse fz = {}) {
    if (need) *need = 0;
    if constexpr (sizeof(T) == 8) {
        return LF_OK;
    } else {
        const T* G = static_cast<const T*>(g);
        const T* Q = static_cast<const T*>(q);
        const T* K = static_cast<const T*>(kT);
        T* DQp = static_cast<T*>(dq);
        T* DKp = static_cast<T*>(dk);
        float* W = static_cast<float*>(ws);
        // configuration-5 channels and landmarks: the 16-warp wide kernel
        if (wide_flat_shape(m, d))
            return launch_bwd_wide_flat<T, 2, 8, 32, 2 * kThreads>(G, Q, K, DQp, DKp, bh, n, m, d, W, ws_bytes, need,
                                                                    st, fz);
        if (!(d <= 32 && m <= 64)) return LF_OK;
        const int64_t m4 = (m + 3) & ~3;
        switch (m4 <= 16 ? 16 : (m4 <= 32 ? 32 : (m4 <= 48 ? 48 : (m4 <= 52 ? 52 : (m4 <= 56 ? 56 : 64))))) {
            case 16: return launch_bwd_flat<T, 16>(G, Q, K, DQp, DKp, bh, n, m, d, W, ws_bytes, need, st, fz);
            case 32: return launch_bwd_flat<T, 32>(G, Q, K, DQp, DKp, bh, n, m, d, W, ws_bytes, need, st, fz);
            case 48: return launch_bwd_flat<T, 48>(G, Q, K, DQp, DKp, bh, n, m, d, W, ws_bytes, need, st, fz);
            case 52: return launch_bwd_flat<T, 52>(G, Q, K, DQp, DKp, bh, n, m, d, W, ws_bytes, need, st, fz);
            case 56: return launch_bwd_flat<T, 56>(G, Q, K, DQp, DKp, bh, n, m, d, W, ws_bytes, need, st, fz);
            default: return launch_bwd_flat<T, 64>(G, Q, K, DQp, DKp, bh, n, m, d, W, ws_bytes, need, st, fz);
        }
    }
}

// Wide variant of the fused backward: d <= 64 and m <= 256 (configuration 5:
// d = 64, m = 256).  Landmarks are padded to MPT = 64 * MCNT; warp w handles
// channel block w % DBT, landmark chunk (w / DBT) % MCNT (64 landmarks) and
// row group w / (DBT * MCNT).  Staging: thread t owns landmark column
// t % MPT of every staged row it loads, so column sums of dS stay in one
// register; row sums go through warp shuffles and a small shared array.  The
// next chunk is prefetched into registers during compute.  dQ partials of the
// landmark chunks and dK partials of the row groups are combined in a fixed
// order (bitwise reproducible); the row-split CTAs of one (b,h) form a
// cluster and add their dK through distributed shared memory.
template <typename T, int DBT, int MCNT, int MB, int NT, bool FLAT, bool KM>
__global__ void __launch_bounds__(NT, 1)
lsub_bwd_wide_kernel(const T* __restrict__ g, const T* __restrict__ q, const T* __restrict__ kT,
                     T* __restrict__ dq, T* __restrict__ dk, BwdGeom geo, float* __restrict__ ws) {
    using A = typename Elem<T>::acc;
    constexpr int MPT = MB * MCNT;             // padded landmarks
    constexpr int CW = 32 * DBT;               // channels per CTA
    constexpr int RG = (NT / 32) / (DBT * MCNT);
    constexpr int RC = 4096 / MPT;             // staged rows per chunk (16 values per thread)
    constexpr int GPT = RC * MPT / NT;   // dS values staged per thread
    constexpr int QPT = RC * CW / NT;    // Q values staged per thread
    constexpr int WPR = MPT / 32;              // warps spanning one staged row
    static_assert(RG >= 1 && GPT >= 1 && QPT >= 1 && NT % MPT == 0, "bad wide backward shape");
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int n = geo.n, m = geo.m, d = geo.d, KSTR = geo.KSTR;
    A* gs = reinterpret_cast<A*>(smem_raw);        // [RC][MPT]
    A* qs = gs + RC * MPT;                          // [RC][CW]
    A* rpart = qs + RC * CW;                        // [RC][WPR]
    A* csum = rpart + RC * WPR;                     // [MPT]
    A* cpart = csum + MPT;                          // [NT / MPT][MPT]
    A* dqp = cpart + (NT / MPT) * MPT;        // [MCNT][RC][CW]
    A* dkb = dqp + MCNT * RC * CW;                  // [CW][KSTR]
    A* dpart = dkb + CW * KSTR;                     // [RG][CW][KSTR] (RG > 1)

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int db = warp % DBT, mcb = (warp / DBT) % MCNT, rg = warp / (DBT * MCNT);
    const int cbase = (int)blockIdx.z * CW;  // channel group of this CTA (grid.z)
    const int cw = min(CW, d - cbase);       // channels of the group
    const int cl = db * 32 + lane, c = cbase + cl;
    const bool lane_active = cl < cw;
    const int j0 = mcb * MB;
    const int sj = tid % MPT, srow0 = tid / MPT;    // staging column / first row
    constexpr int SRS = NT / MPT;             // staging row stride

    // FLAT: this CTA walks a contiguous run of P 64-row units of the flattened
    // (b,h) x rows space, one segment per (b,h) it touches; otherwise one
    // segment: rows [x * rows_per_cta, ...) of (b,h) = blockIdx.y.
    int64_t u = FLAT ? (int64_t)blockIdx.x * geo.P : 0;
    const int64_t u_end = FLAT ? ((u + geo.P < geo.total) ? u + geo.P : geo.total) : 1;
    for (int seg = 0; u < u_end; ++seg) {
    int bh;
    int64_t r_begin, r_end, u_next;
    if constexpr (FLAT) {
        bh = (int)(u / geo.U);
        const int64_t ub = (int64_t)bh * geo.U;
        u_next = (ub + geo.U < u_end) ? ub + geo.U : u_end;
        r_begin = (u - ub) * kRowChunk;
        r_end = (u_next - ub) * kRowChunk;
        if (r_end > n) r_end = n;
    } else {
        bh = blockIdx.y;
        r_begin = (int64_t)blockIdx.x * geo.rows_per_cta;
        r_end = (r_begin + geo.rows_per_cta < (int64_t)n) ? r_begin + geo.rows_per_cta : (int64_t)n;
        u_next = 1;
    }
    const T* Gb = g + (int64_t)bh * n * m;
    const T* Qb = q + (int64_t)bh * n * d;
    const T* Kb = kT + (int64_t)bh * d * m;

    A kreg[MB], dka[MB];
#pragma unroll
    for (int jj = 0; jj < MB; ++jj) {
        const int j = j0 + jj;
        kreg[jj] = (lane_active && j < m) ? Elem<T>::load(Kb[(int64_t)c * m + j]) : A(0);
        dka[jj] = A(0);
    }
    A colacc = A(0);


    A pg[GPT], pq[QPT];
    auto load_chunk = [&](int64_t rc) {
#pragma unroll
        for (int k = 0; k < GPT; ++k) {
            const int64_t row = rc + srow0 + SRS * k;
            if constexpr (KM)
                pg[k] = (row < r_end && sj < m)
                            ? grad_at<T>(Gb, static_cast<const T*>(geo.km) + (Gb - g), geo.kscale, row * m + sj)
                            : A(0);
            else
                pg[k] = (row < r_end && sj < m) ? Elem<T>::load(Gb[row * m + sj]) : A(0);
        }
#pragma unroll
        for (int k = 0; k < QPT; ++k) {
            const int e = tid + NT * k;
            const int i = e / CW, x = e % CW;
            const int64_t row = rc + i;
            pq[k] = (row < r_end && x < cw) ? Elem<T>::load(Qb[row * d + cbase + x]) : A(0);
        }
    };
    if (r_begin < r_end) load_chunk(r_begin);

    for (int64_t rc = r_begin; rc < r_end; rc += RC) {
        const int rows = (int)((r_end - rc) < RC ? (r_end - rc) : RC);
        __syncthreads();  // previous chunk fully consumed
#pragma unroll
        for (int k = 0; k < GPT; ++k) {
            const int i = srow0 + SRS * k;
            gs[i * MPT + sj] = pg[k];
            colacc += pg[k];
            A rs = pg[k];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, o);
            if (lane == 0) rpart[i * WPR + (sj >> 5)] = rs;
        }
#pragma unroll
        for (int k = 0; k < QPT; ++k) qs[tid + NT * k] = pq[k];
        __syncthreads();
        if (rc + RC < r_end) load_chunk(rc + RC);

        if (lane_active) {
#pragma unroll 1
            for (int i = rg; i < rows; i += RG) {
                const A qv = qs[i * CW + cl];
                const A* grow = gs + i * MPT + j0;
                A dqa = A(0);
                [[maybe_unused]] float dq4[4] = {0.f, 0.f, 0.f, 0.f};
                [[maybe_unused]] unsigned long long qq = 0;
                if constexpr (sizeof(A) == 4) asm("mov.b64 %0, {%1, %1};" : "=l"(qq) : "f"(qv));
#pragma unroll
                for (int j4 = 0; j4 < MB; j4 += 4) {
                    A gv[4];
                    if constexpr (sizeof(A) == 4) {
                        float4 t4 = *reinterpret_cast<const float4*>(grow + j4);
                        gv[0] = t4.x; gv[1] = t4.y; gv[2] = t4.z; gv[3] = t4.w;
                        bwd_quad_x2(qq, kreg[j4], kreg[j4 + 1], kreg[j4 + 2], kreg[j4 + 3], gv, dq4,
                                    dka[j4], dka[j4 + 1], dka[j4 + 2], dka[j4 + 3]);
                    } else {
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            gv[e] = grow[j4 + e];
                            const A t = step_of<A>(qv, kreg[j4 + e]);
                            dqa = fma_acc(gv[e], t, dqa);
                            dka[j4 + e] = fma_acc(gv[e], t, dka[j4 + e]);
                        }
                    }
                }
                if constexpr (sizeof(A) == 4) dqa = (dq4[0] + dq4[1]) + (dq4[2] + dq4[3]);
                dqp[(mcb * RC + i) * CW + cl] = dqa;
            }
        }
        __syncthreads();
        // dQ = 2 * sum over landmark chunks (fixed order) - row sum of dS
        for (int e = tid; e < rows * CW; e += NT) {
            const int i = e / CW, x = e % CW;
            if (x >= cw) continue;
            A acc = A(0);
#pragma unroll
            for (int b = 0; b < MCNT; ++b) acc += dqp[(b * RC + i) * CW + x];
            A rs = A(0);
#pragma unroll
            for (int w = 0; w < WPR; ++w) rs += rpart[i * WPR + w];
            const T v = Elem<T>::store(A(2) * acc - rs);
            const int64_t o = ((int64_t)bh * n + rc + i) * d + cbase + x;
            dq[o] = v;
            for (int p = 0; p < geo.ndqx; ++p) static_cast<T*>(geo.dqx[p])[o] = v;  // peer gather buffers
        }
    }

    // Column sums of dS over the CTA's rows, then dKT = csum - 2 sum g*t.
    cpart[srow0 * MPT + sj] = colacc;
    if (lane_active) {
#pragma unroll
        for (int jj = 0; jj < MB; ++jj) {
            const int j = j0 + jj;
            if (j < m) {
                if (RG == 1) dkb[cl * KSTR + j] = A(-2) * dka[jj];
                else dpart[(rg * CW + cl) * KSTR + j] = A(-2) * dka[jj];
            }
        }
    }
    __syncthreads();
    for (int j = tid; j < m; j += NT) {
        A s = A(0);
        for (int r = 0; r < SRS; ++r) s += cpart[r * MPT + j];
        csum[j] = s;
    }
    __syncthreads();
    for (int e = tid; e < CW * m; e += NT) {
        const int cc = e / m, j = e % m;
        if (cc >= cw) continue;
        A s = csum[j];
        if (RG == 1) {
            s += dkb[cc * KSTR + j];
        } else {
            for (int r = 0; r < RG; ++r) s += dpart[(r * CW + cc) * KSTR + j];
        }
        dkb[cc * KSTR + j] = s;
    }
    if constexpr (FLAT) {
        // A (b,h) wholly inside this CTA gets its dK^T directly; the part of a
        // (b,h) shared with other CTAs goes to slot 2*CTA (first segment) or
        // 2*CTA+1 (last), summed in CTA order by lsub_bwd_dk_finalize.
        const bool whole = (u == (int64_t)bh * geo.U) && (u_next == (int64_t)bh * geo.U + geo.U);
        T* dkout = dk + ((int64_t)bh * d + cbase) * m;
        float* slot = ws + ((int64_t)2 * blockIdx.x + (seg == 0 ? 0 : 1)) * d * m + (int64_t)cbase * m;
        for (int e = tid; e < cw * m; e += NT) {
            const int cc = e / m, j = e - cc * m;
            const A v = dkb[cc * KSTR + j];
            if (whole) dkout[e] = Elem<T>::store(v);
            else slot[e] = (float)v;
        }
        __syncthreads();  // the shared buffers are reused by the next segment
        u = u_next;
    } else {
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    const int cs = (int)cluster.num_blocks();
    const int rank = (int)cluster.block_rank();
    const int total = cw * m;
    const int per = (total + cs - 1) / cs;
    const int e0 = rank * per, e1 = min(total, e0 + per);
    T* dkout = dk + ((int64_t)bh * d + cbase) * m;
    for (int e = e0 + tid; e < e1; e += NT) {
        const int cc = e / m, j = e - cc * m;
        A s = A(0);
        for (int r = 0; r < cs; ++r) {
            const A* peer = cluster.map_shared_rank(dkb, r);
            s += peer[cc * KSTR + j];
        }
        dkout[e] = Elem<T>::store(s);
    }
    cluster.sync();
    u = u_next;
    }
    }  // segments
}

template <typename T, int DBT, int MCNT, int MB = 64, int NT = kThreads>
int launch_bwd_wide(const T* g, const T* q, const T* kT, T* dq, T* dk, int64_t bh, int64_t n, int64_t m,
                    int64_t d, cudaStream_t st, GFuse fz = {}) {
    using A = typename Elem<T>::acc;
    constexpr int MPT = MB * MCNT, CW = 32 * DBT, RG = (NT / 32) / (DBT * MCNT), RC = 4096 / MPT;
    BwdGeom geo;
    geo.n = (int)n; geo.m = (int)m; geo.d = (int)d;
    geo.km = fz.km; geo.kscale = fz.kscale;
    geo.DBC = DBT; geo.MCN = MCNT; geo.RG = RG; geo.MP = MPT; geo.RC = RC;
    geo.KSTR = (int)(m | 1);
    size_t smem = sizeof(A) * ((size_t)RC * MPT + (size_t)RC * CW + (size_t)RC * (MPT / 32) + MPT +
                               (size_t)(NT / MPT) * MPT + (size_t)MCNT * RC * CW + (size_t)CW * geo.KSTR +
                               (RG > 1 ? (size_t)RG * CW * geo.KSTR : 0));
    if (smem > (size_t)max_optin_smem()) {
        set_error("LaplaceSubtraction backward: needs %zu bytes of shared memory", smem);
        return LF_ERR_UNSUPPORTED;
    }
    auto kern = fz.km ? lsub_bwd_wide_kernel<T, DBT, MCNT, MB, NT, false, true>
                      : lsub_bwd_wide_kernel<T, DBT, MCNT, MB, NT, false, false>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const int64_t slots = cta_slots(kern, smem, NT);
    const int64_t max_by_rows = (n + RC - 1) / RC;
    (void)slots;
    const int64_t groups = (d + CW - 1) / CW;  // channel groups over grid.z
    // Cluster size: the CTAs of one (b,h) split its rows and form a cluster,
    // so a cluster must fit in one GPC.  For each size the driver reports how
    // many such clusters run at once; the estimated time is the number of
    // waves times the rows per CTA.  Sizes above 8 (non-portable) help when
    // there are few (b,h) per GPU (configuration 5 over 8 GPUs: 16).
    int cmax = 8;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) cmax = 16;
    else cudaGetLastError();
    int64_t cs = 1;
    double best_t = -1.0;
    for (int c = 1; c <= cmax && c <= (max_by_rows < 1 ? 1 : max_by_rows); ++c) {
        const int clusters = active_clusters(kern, c, NT, smem);
        if (clusters < 1) continue;
        const double waves = (double)((bh * groups + clusters - 1) / clusters);
        const double t = waves * (double)((n + c - 1) / c);
        if (best_t < 0.0 || t < best_t * (1.0 - 1e-9)) { best_t = t; cs = c; }
    }
    int64_t rpc = (n + cs - 1) / cs;
    rpc = ((rpc + RC - 1) / RC) * RC;
    geo.rows_per_cta = (int)rpc;
    if (bh > 65535) { set_error("b*h = %lld exceeds 65535", (long long)bh); return LF_ERR_UNSUPPORTED; }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)cs, (unsigned)bh, (unsigned)groups);
    cfg.blockDim = dim3(NT, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t err = cudaLaunchKernelEx(&cfg, kern, g, q, kT, dq, dk, geo, static_cast<float*>(nullptr));
    if (err != cudaSuccess) {
        set_error("lsub_bwd_wide_kernel launch: %s", cudaGetErrorString(err));
        return LF_ERR_CUDA;
    }
    return check_launch("lsub_bwd_wide_kernel");
}

// Balanced launch of the wide backward (both gradients, workspace): every CTA
// slot of the GPU takes a contiguous run of P 64-row units of all (b,h)
// (lf_laplace_sub_bwd_ws), as for the fast kernel; the dKT partials of a
// (b,h) shared by several CTAs are summed by lsub_bwd_dk_finalize.
template <typename T, int DBT, int MCNT, int MB, int NT>
int launch_bwd_wide_flat(const T* g, const T* q, const T* kT, T* dq, T* dk, int64_t bh, int64_t n, int64_t m,
                         int64_t d, float* ws, size_t ws_bytes, size_t* need, cudaStream_t st, GFuse fz) {
    using A = typename Elem<T>::acc;
    constexpr int MPT = MB * MCNT, CW = 32 * DBT, RG = (NT / 32) / (DBT * MCNT), RC = 4096 / MPT;
    BwdGeom geo;
    geo.n = (int)n; geo.m = (int)m; geo.d = (int)d;
    geo.km = fz.km; geo.kscale = fz.kscale;
    if (fz.ndqx < 0 || fz.ndqx > LF_MAX_PEERS) { set_error("at most %d dQ peers", LF_MAX_PEERS); return LF_ERR_INVALID; }
    geo.ndqx = fz.ndqx;
    for (int p = 0; p < fz.ndqx; ++p) geo.dqx[p] = fz.dqx[p];
    geo.DBC = DBT; geo.MCN = MCNT; geo.RG = RG; geo.MP = MPT; geo.RC = RC;
    geo.KSTR = (int)(m | 1);
    geo.rows_per_cta = 0;
    size_t smem = sizeof(A) * ((size_t)RC * MPT + (size_t)RC * CW + (size_t)RC * (MPT / 32) + MPT +
                               (size_t)(NT / MPT) * MPT + (size_t)MCNT * RC * CW + (size_t)CW * geo.KSTR +
                               (RG > 1 ? (size_t)RG * CW * geo.KSTR : 0));
    if (smem > (size_t)max_optin_smem()) {
        set_error("LaplaceSubtraction backward: needs %zu bytes of shared memory", smem);
        return LF_ERR_UNSUPPORTED;
    }
    auto kern = fz.km ? lsub_bwd_wide_kernel<T, DBT, MCNT, MB, NT, true, true>
                      : lsub_bwd_wide_kernel<T, DBT, MCNT, MB, NT, true, false>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const int64_t slots = cta_slots(kern, smem, NT);
    geo.U = (n + kRowChunk - 1) / kRowChunk;
    geo.total = bh * geo.U;
    geo.P = (geo.total + slots - 1) / slots;
    const int64_t grid = (geo.total + geo.P - 1) / geo.P;
    const size_t bytes = (size_t)2 * grid * d * m * sizeof(float);
    if (need) *need = bytes;
    if (!ws) return LF_OK;
    if (ws_bytes < bytes) {
        set_error("LaplaceSubtraction backward: workspace of %zu bytes, %zu needed", ws_bytes, bytes);
        return LF_ERR_INVALID;
    }
    kern<<<(unsigned)grid, NT, smem, st>>>(g, q, kT, dq, dk, geo, ws);
    int rc = check_launch("lsub_bwd_wide_kernel");
    if (rc) return rc;
    if (bh > 0x7fffffff) { set_error("b*h too large"); return LF_ERR_UNSUPPORTED; }
    const unsigned eblocks = (unsigned)((d * m + kThreads - 1) / kThreads);
    lsub_bwd_dk_finalize<T><<<dim3((unsigned)bh, eblocks, 1), kThreads, 0, st>>>(ws, dk, (int)d, (int)m, geo.U, geo.P);
    return check_launch("lsub_bwd_dk_finalize");
}

// Landmark chunk per warp (MB) and number of chunks (mcn): least padding of m
// with at most 8 chunks; ties prefer chunks of at most 52 landmarks (larger
// ones spill registers in the fused kernel), then the larger chunk.
int pick_mb(int64_t m, int& mcn) {
    static const int cands[] = {8, 16, 24, 32, 40, 48, 52, 56, 64};
    int best = 0;
    int64_t best_pad = -1;
    for (int c : cands) {
        int64_t chunks = (m + c - 1) / c;
        if (chunks > kThreads / 32) continue;
        int64_t pad = chunks * c;
        bool better = best_pad < 0 || pad < best_pad;
        if (!better && pad == best_pad) {
            bool c_ok = c <= 52, b_ok = best <= 52;
            better = (c_ok && !b_ok) || (c_ok == b_ok && c > best);
        }
        if (better) { best = c; best_pad = pad; }
    }
    mcn = best ? (int)((m + best - 1) / best) : 0;
    return best;
}

template <typename T, int MB, bool DQ, bool DK, int MINB>
int launch_bwd_mb(const T* g, const T* q, const T* kT, T* dq, T* dk, int64_t bh, int64_t n,
                  int64_t m, int64_t d, int mcn, cudaStream_t st, GFuse fz = {}) {
    using A = typename Elem<T>::acc;
    BwdGeom geo;
    geo.n = (int)n; geo.m = (int)m; geo.d = (int)d;
    geo.km = fz.km; geo.kscale = fz.kscale;
    const int DB = (int)((d + 31) / 32);
    geo.MCN = mcn;
    geo.DBC = (kThreads / 32) / mcn;
    if (geo.DBC > DB) geo.DBC = DB;
    if (geo.DBC < 1) geo.DBC = 1;
    const int64_t dgroups = (DB + geo.DBC - 1) / geo.DBC;
    geo.RG = (kThreads / 32) / (geo.DBC * geo.MCN);
    geo.MP = (int)(((m + 3) / 4) * 4);
    if (geo.MP < mcn * MB) geo.MP = mcn * MB;
    geo.KSTR = (int)(m | 1);
    const int CW = geo.DBC * 32;
    auto smem_for = [&](int rc) {
        return sizeof(A) * ((size_t)rc * geo.MP + (size_t)rc * CW + rc + (geo.MCN > 1 ? (size_t)rc * CW : 0) +
                            geo.MP + (DK ? (size_t)CW * geo.KSTR + (size_t)(kThreads / 32) * geo.MP : 0));
    };
    geo.RC = kRowChunk;
    while (geo.RC > 8 && smem_for(geo.RC) > (size_t)max_optin_smem()) geo.RC /= 2;
    size_t smem = smem_for(geo.RC);
    if (smem > (size_t)max_optin_smem()) {
        set_error("LaplaceSubtraction backward: needs %zu bytes of shared memory", smem);
        return LF_ERR_UNSUPPORTED;
    }
    auto kern = lsub_bwd_kernel<T, MB, DQ, DK, MINB>;
    if (smem > 48 * 1024)
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    // Split each (b,h) over a cluster of cs <= 8 CTAs along the rows; cs is
    // chosen so that the CTAs fill whole waves of the machine's CTA slots
    // (ties: fewer CTAs per cluster).
    const int64_t units = bh * dgroups;
    const int64_t slots = cta_slots(kern, smem);
    const int64_t max_by_rows = (n + geo.RC - 1) / geo.RC;
    int64_t cs = 1;
    double best = -1.0;
    for (int64_t c = 1; c <= 8 && c <= (max_by_rows < 1 ? 1 : max_by_rows); ++c) {
        double eff = wave_efficiency(units * c, slots);
        if (eff > best + 1e-9) { best = eff; cs = c; }
    }
    int64_t rpc = (n + cs - 1) / cs;
    rpc = ((rpc + geo.RC - 1) / geo.RC) * geo.RC;
    geo.rows_per_cta = (int)rpc;
    if (bh > 65535 || dgroups > 65535) { set_error("b*h = %lld exceeds 65535", (long long)bh); return LF_ERR_UNSUPPORTED; }

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)cs, (unsigned)bh, (unsigned)dgroups);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t err = cudaLaunchKernelEx(&cfg, kern, g, q, kT, dq, dk, geo);
    if (err != cudaSuccess) {
        set_error("lsub_bwd_kernel launch: %s", cudaGetErrorString(err));
        return LF_ERR_CUDA;
    }
    return check_launch("lsub_bwd_kernel");
}

template <typename T, bool DQ, bool DK>
int launch_bwd_t(const void* g, const void* q, const void* kT, void* dq, void* dk, int64_t bh,
                 int64_t n, int64_t m, int64_t d, cudaStream_t st, GFuse fz = {}) {
    const T* G = static_cast<const T*>(g);
    const T* Q = static_cast<const T*>(q);
    const T* K = static_cast<const T*>(kT);
    T* DQp = static_cast<T*>(dq);
    T* DKp = static_cast<T*>(dk);
    if constexpr (sizeof(T) != 8) {
        // fast path: one channel block, one landmark chunk of 4..64 (multiple of 4)
        if (d <= 32 && m <= 64) {
            const int64_t m4 = (m + 3) & ~3;
            switch (m4 <= 16 ? 16 : (m4 <= 32 ? 32 : (m4 <= 48 ? 48 : (m4 <= 52 ? 52 : (m4 <= 56 ? 56 : 64))))) {
                case 16: return launch_bwd_fast<T, 16, DQ, DK>(G, Q, K, DQp, DKp, bh, n, m, d, st, fz);
                case 32: return launch_bwd_fast<T, 32, DQ, DK>(G, Q, K, DQp, DKp, bh, n, m, d, st, fz);
                case 48: return launch_bwd_fast<T, 48, DQ, DK>(G, Q, K, DQp, DKp, bh, n, m, d, st, fz);
                case 52: return launch_bwd_fast<T, 52, DQ, DK>(G, Q, K, DQp, DKp, bh, n, m, d, st, fz);
                case 56: return launch_bwd_fast<T, 56, DQ, DK>(G, Q, K, DQp, DKp, bh, n, m, d, st, fz);
                default: return launch_bwd_fast<T, 64, DQ, DK>(G, Q, K, DQp, DKp, bh, n, m, d, st, fz);
            }
        }
    }
    if constexpr (sizeof(T) != 8) {
        // wide path (both gradients): d <= 64, 64 < m <= 256 or 32 < d <= 64
        if (DQ && DK && d <= 64 && m <= 256 && (m > 64 || d > 32)) {
            const int mc = m <= 64 ? 1 : (m <= 128 ? 2 : 4);
            if (d <= 32) {
                if (mc == 2) return launch_bwd_wide<T, 1, 2>(G, Q, K, DQp, DKp, bh, n, m, d, st, fz);
                return launch_bwd_wide<T, 1, 4>(G, Q, K, DQp, DKp, bh, n, m, d, st, fz);
            }
            if (mc == 1) return launch_bwd_wide<T, 2, 1>(G, Q, K, DQp, DKp, bh, n, m, d, st, fz);
            if (mc == 2) return launch_bwd_wide<T, 2, 2>(G, Q, K, DQp, DKp, bh, n, m, d, st, fz);
            // 128 < m <= 256: 32 landmarks per warp, 16 warps (half the
            // registers per thread of 64-landmark warps, twice the warps per SM)
            return launch_bwd_wide<T, 2, 8, 32, 2 * kThreads>(G, Q, K, DQp, DKp, bh, n, m, d, st, fz);
        }
    }
    int mcn = 1;
    int mb = pick_mb(m, mcn);
    if (mb == 0) {
        set_error("LaplaceSubtraction backward supports m <= 512 (got %lld)", (long long)m);
        return LF_ERR_UNSUPPORTED;
    }
    constexpr int kMinb = (DQ && sizeof(T) != 8) ? 2 : 1;
#define LF_BWD_CASE(MBV)                                                                              \
    case MBV:                                                                                         \
        return launch_bwd_mb<T, MBV, DQ, DK, kMinb>(G, Q, K, DQp, DKp, bh, n, m, d, mcn, st, fz);
    switch (mb) {
        LF_BWD_CASE(8) LF_BWD_CASE(16) LF_BWD_CASE(24) LF_BWD_CASE(32) LF_BWD_CASE(40)
        LF_BWD_CASE(48) LF_BWD_CASE(52) LF_BWD_CASE(56) LF_BWD_CASE(64)
        default: break;
    }
#undef LF_BWD_CASE
    set_error("internal: no backward tile for m=%lld", (long long)m);
    return LF_ERR_UNSUPPORTED;
}

// ---------------------------------------------------------------------------
// Legacy reduce forward: one warp per output.  Partials follow the
// reference's thread assignment for blockDim b = min(d, 256) (thread t sums
// channels t, t+b, ... in the storage type) and its halving tree
// s[t] += s[t+stride], stride = b/2, b/4, ..., including the partials the
// tree drops when b is not a power of two (:429-442).
// ---------------------------------------------------------------------------
template <typename T>
struct StoreArith {  // one operation in float, rounded to T (c10::Half semantics)
    static __device__ __forceinline__ T add(T a, T b) { return T(float(a) + float(b)); }
    static __device__ __forceinline__ T sub(T a, T b) { return T(float(a) - float(b)); }
    static __device__ __forceinline__ bool nonneg(T a) { return float(a) >= 0.f; }
    static __device__ __forceinline__ T neg(T a) { return T(-float(a)); }
};
template <> struct StoreArith<float> {
    static __device__ __forceinline__ float add(float a, float b) { float r; asm("add.rn.ftz.f32 %0,%1,%2;" : "=f"(r) : "f"(a), "f"(b)); return r; }
    static __device__ __forceinline__ float sub(float a, float b) { return sub_ftz(a, b); }
    static __device__ __forceinline__ bool nonneg(float a) { return a >= 0.f; }
    static __device__ __forceinline__ float neg(float a) { return -a; }
};
template <> struct StoreArith<double> {
    static __device__ __forceinline__ double add(double a, double b) { return __dadd_rn(a, b); }
    static __device__ __forceinline__ double sub(double a, double b) { return __dsub_rn(a, b); }
    static __device__ __forceinline__ bool nonneg(double a) { return a >= 0.0; }
    static __device__ __forceinline__ double neg(double a) { return -a; }
};

template <typename T>
__global__ void __launch_bounds__(kThreads)
lsub_reduce_kernel(const T* __restrict__ q, const T* __restrict__ kT, T* __restrict__ s,
                   int64_t total, int n, int m, int d) {
    __shared__ T part[kThreads / 32][256];
    using Ar = StoreArith<T>;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = d < 256 ? d : 256;
    T* sp = part[warp];
    for (int64_t o = (int64_t)blockIdx.x * (kThreads / 32) + warp; o < total;
         o += (int64_t)gridDim.x * (kThreads / 32)) {
        const int64_t per_bh = (int64_t)n * m;
        const int64_t bhi = o / per_bh;
        const int64_t rem = o - bhi * per_bh;
        const int i = (int)(rem / m), j = (int)(rem - (int64_t)(rem / m) * m);
        const T* qr = q + (bhi * n + i) * d;
        const T* kb = kT + bhi * (int64_t)d * m;
        for (int t = lane; t < b; t += 32) {
            T acc = T(0.f);
            for (int cc = t; cc < d; cc += b) {
                T diff = Ar::sub(qr[cc], kb[(int64_t)cc * m + j]);
                acc = Ar::add(acc, Ar::nonneg(diff) ? diff : Ar::neg(diff));
            }
            sp[t] = acc;
        }
        __syncwarp();
        for (int stride = b / 2; stride > 0; stride >>= 1) {
            for (int t = lane; t < stride; t += 32) sp[t] = Ar::add(sp[t], sp[t + stride]);
            __syncwarp();
        }
        if (lane == 0) s[o] = sp[0];
        __syncwarp();
    }
}

int check_args(const void* a, const void* b, const void* c, int64_t bh, int64_t n, int64_t m,
               int64_t d, int dtype) {
    if (dtype_size(dtype) == 0) { set_error("unsupported dtype code %d", dtype); return LF_ERR_DTYPE; }
    if (bh < 0 || n < 0 || m < 0 || d < 0) { set_error("negative size"); return LF_ERR_INVALID; }
    if (n > 0x7fffffffLL || m > 0x7fffffffLL || d > 0x7fffffffLL) {
        set_error("sizes must fit in 31 bits per dimension"); return LF_ERR_UNSUPPORTED;
    }
    if ((bh > 0 && n > 0 && m > 0 && d > 0) && (!a || !b || !c)) { set_error("null pointer"); return LF_ERR_INVALID; }
    return LF_OK;
}

}  // namespace
}  // namespace lfb

using namespace lfb;

extern "C" int lf_laplace_sub_fwd(const void* q, const void* kT, void* s, int64_t bh, int64_t n,
                                  int64_t m, int64_t d, int dtype, lf_stream_t stream) {
    clear_error();
    int rc = check_args(q, kT, s, bh, n, m, d, dtype);
    if (rc) return rc;
    if (bh == 0 || n == 0 || m == 0) return LF_OK;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (d == 0) {
        if (cudaMemsetAsync(s, 0, (size_t)(bh * n * m) * dtype_size(dtype), st) != cudaSuccess)
            return check_launch("memset");
        return LF_OK;
    }
    LF_DISPATCH(dtype, T, return launch_fwd<T>(q, kT, s, bh, n, m, d, st));
    return LF_OK;
}

template <typename T>
__global__ void fill_one_kernel(T* p, int64_t count) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x)
        p[i] = Elem<T>::store(typename Elem<T>::acc(1));
}

extern "C" int lf_laplace_kernel_fwd(const void* q, const void* kT, void* kmat, int64_t bh, int64_t n, int64_t m,
                                     int64_t d, int dtype, double scale, lf_stream_t stream) {
    clear_error();
    int rc = check_args(q, kT, kmat, bh, n, m, d, dtype);
    if (rc) return rc;
    if (!(scale == scale) || scale > 3.0e38 || scale < -3.0e38) {
        set_error("lf_laplace_kernel_fwd: scale must be finite");
        return LF_ERR_INVALID;
    }
    if (bh == 0 || n == 0 || m == 0) return LF_OK;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (d == 0) {  // S = 0, exp(0) = 1
        const int64_t count = bh * n * m;
        int64_t blocks = (count + kThreads - 1) / kThreads;
        if (blocks > (int64_t)num_sms() * 8) blocks = (int64_t)num_sms() * 8;
        LF_DISPATCH(dtype, T, {
            fill_one_kernel<T><<<(unsigned)blocks, kThreads, 0, st>>>(static_cast<T*>(kmat), count);
            return check_launch("fill_one_kernel");
        });
        return LF_OK;
    }
    LF_DISPATCH(dtype, T, return launch_fwd<T>(q, kT, kmat, bh, n, m, d, st, scale, true));
    return LF_OK;
}

static int bwd_common(const void* g, const void* q, const void* kT, void* dq, void* dk, int64_t bh,
                      int64_t n, int64_t m, int64_t d, int dtype, lf_stream_t stream, GFuse fz = {}) {
    int rc = check_args(g, q, kT, bh, n, m, d, dtype);
    if (rc) return rc;
    if (!dq && !dk) return LF_OK;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (bh == 0 || d == 0) return LF_OK;
    if (n == 0 || m == 0) {  // empty reductions: gradients are zero
        size_t es = dtype_size(dtype);
        if (dq && cudaMemsetAsync(dq, 0, (size_t)(bh * n * d) * es, st) != cudaSuccess) return check_launch("memset");
        if (dk && cudaMemsetAsync(dk, 0, (size_t)(bh * d * m) * es, st) != cudaSuccess) return check_launch("memset");
        return LF_OK;
    }
    if (dq && dk) { LF_DISPATCH(dtype, T, return launch_bwd_t<T, true, true>(g, q, kT, dq, dk, bh, n, m, d, st, fz)); }
    if (dq) { LF_DISPATCH(dtype, T, return launch_bwd_t<T, true, false>(g, q, kT, dq, dk, bh, n, m, d, st, fz)); }
    LF_DISPATCH(dtype, T, return launch_bwd_t<T, false, true>(g, q, kT, dq, dk, bh, n, m, d, st, fz));
    return LF_OK;
}

extern "C" int lf_laplace_sub_bwd(const void* g, const void* q, const void* kT, void* dq, void* dkT,
                                  int64_t bh, int64_t n, int64_t m, int64_t d, int dtype,
                                  lf_stream_t stream) {
    clear_error();
    return bwd_common(g, q, kT, dq, dkT, bh, n, m, d, dtype, stream);
}

// Workspace bytes of lf_laplace_sub_bwd_ws for this shape (0: the shape
// runs without workspace).  Depends on the current device's SM count.
extern "C" size_t lf_laplace_sub_bwd_workspace_size(int64_t bh, int64_t n, int64_t m, int64_t d, int dtype) {
    clear_error();
    if (bh <= 0 || n <= 0 || m <= 0 || d <= 0) return 0;
    if (dtype < LF_F32 || dtype > LF_BF16) { set_error("unsupported dtype code %d", dtype); return 0; }
    size_t need = 0;
    LF_DISPATCH(dtype, T, {
        launch_bwd_flat_t<T>(nullptr, nullptr, nullptr, nullptr, nullptr, bh, n, m, d, nullptr, 0, &need, 0);
        return need;
    });
    return 0;
}

extern "C" int lf_laplace_sub_bwd_ws(const void* g, const void* q, const void* kT, void* dq, void* dkT,
                                     int64_t bh, int64_t n, int64_t m, int64_t d, int dtype, void* workspace,
                                     size_t workspace_bytes, lf_stream_t stream) {
    clear_error();
    const size_t need = lf_laplace_sub_bwd_workspace_size(bh, n, m, d, dtype);
    if (need == 0 || !dq || !dkT) return bwd_common(g, q, kT, dq, dkT, bh, n, m, d, dtype, stream);
    int rc = check_args(g, q, kT, bh, n, m, d, dtype);
    if (rc) return rc;
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 15)) {
        set_error("LaplaceSubtraction backward: workspace must be a 16-byte aligned device pointer");
        return LF_ERR_INVALID;
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    LF_DISPATCH(dtype, T, return launch_bwd_flat_t<T>(g, q, kT, dq, dkT, bh, n, m, d, workspace, workspace_bytes,
                                                      nullptr, st));
    return LF_OK;
}

// lf_laplace_sub_bwd_ws with dQ also stored into peer gather buffers: from
// inside the balanced wide kernel where it runs, else by a put afterwards.
extern "C" int lf_laplace_sub_bwd_peers(const void* g, const void* q, const void* kT, void* dq, void* dkT,
                                        void* const* dq_peers, int npeer, int64_t bh, int64_t n, int64_t m,
                                        int64_t d, int dtype, void* workspace, size_t workspace_bytes,
                                        lf_stream_t stream) {
    clear_error();
    if (npeer < 0 || npeer > LF_MAX_PEERS || (npeer > 0 && !dq_peers)) {
        set_error("lf_laplace_sub_bwd_peers: %d peers (at most %d, table required)", npeer, LF_MAX_PEERS);
        return LF_ERR_INVALID;
    }
    for (int p = 0; p < npeer; ++p)
        if (!dq_peers[p]) { set_error("lf_laplace_sub_bwd_peers: null peer %d", p); return LF_ERR_INVALID; }
    if (!dq || !dkT) { set_error("lf_laplace_sub_bwd_peers: dq and dkT are required"); return LF_ERR_INVALID; }
    const size_t need = lf_laplace_sub_bwd_workspace_size(bh, n, m, d, dtype);
    if (npeer > 0 && need > 0 && wide_flat_shape(m, d) && dtype != LF_F64) {
        int rc = check_args(g, q, kT, bh, n, m, d, dtype);
        if (rc) return rc;
        if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 15)) {
            set_error("LaplaceSubtraction backward: workspace must be a 16-byte aligned device pointer");
            return LF_ERR_INVALID;
        }
        GFuse fz;
        fz.dqx = dq_peers;
        fz.ndqx = npeer;
        cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
        LF_DISPATCH(dtype, T, return launch_bwd_flat_t<T>(g, q, kT, dq, dkT, bh, n, m, d, workspace, workspace_bytes,
                                                          nullptr, st, fz));
        return LF_OK;
    }
    int rc = lf_laplace_sub_bwd_ws(g, q, kT, dq, dkT, bh, n, m, d, dtype, workspace, workspace_bytes, stream);
    if (rc || npeer == 0) return rc;
    return lf_peer_put(dq, (size_t)(bh * n * d) * dtype_size(dtype), dq_peers, npeer, stream);
}

// Gradients of Kmat = exp(scale * S) (lf_laplace_kernel_fwd) from dKmat, with
// dS = scale * Kmat * dKmat formed while the backward stages its gradient
// tile: no dS tensor is written or read.
extern "C" int lf_laplace_kernel_bwd(const void* gk, const void* kmat, const void* q, const void* kT, void* dq,
                                     void* dkT, int64_t bh, int64_t n, int64_t m, int64_t d, int dtype, double scale,
                                     void* workspace, size_t workspace_bytes, lf_stream_t stream) {
    clear_error();
    if (!kmat && bh * n * m > 0) { set_error("null kmat"); return LF_ERR_INVALID; }
    GFuse fz;
    fz.km = kmat;
    fz.kscale = (float)scale;
    const size_t need = (dq && dkT && workspace) ? lf_laplace_sub_bwd_workspace_size(bh, n, m, d, dtype) : 0;
    if (need == 0) return bwd_common(gk, q, kT, dq, dkT, bh, n, m, d, dtype, stream, fz);
    int rc = check_args(gk, q, kT, bh, n, m, d, dtype);
    if (rc) return rc;
    if (reinterpret_cast<uintptr_t>(workspace) & 15) {
        set_error("LaplaceKernel backward: workspace must be a 16-byte aligned device pointer");
        return LF_ERR_INVALID;
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    LF_DISPATCH(dtype, T, return launch_bwd_flat_t<T>(gk, q, kT, dq, dkT, bh, n, m, d, workspace, workspace_bytes,
                                                      nullptr, st, fz));
    return LF_OK;
}

// ---------------------------------------------------------------------------
// Fused backward without any allocation
// ---------------------------------------------------------------------------
// Scratch of lf_laplace_sub_bwd_noalloc: the dKT partial slots of the
// balanced backward.  A file-scope device array, so it exists on every GPU
// that loads this library from load until process exit, and no call has to
// allocate.  Every call overwrites the slots it later reads, so nothing in
// it has to start at zero; all calls share it, so calls that can overlap on
// the GPU (other streams, other host threads) race on it.
constexpr size_t kNoAllocScratchBytes = (size_t)2 << 20;  // 2 MiB
static __device__ __align__(256) float g_bwd_scratch[kNoAllocScratchBytes / sizeof(float)];

namespace {
constexpr int kNoAllocMaxDev = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kNoAllocMaxDev];

// In host code g_bwd_scratch names a host-side stand-in; the device address
// is asked for with the device current.  Only a successful lookup is kept, so
// a failure (for example a first call made during stream capture) is
// reported and the next call tries again.
void* scratch_address(int dev, cudaError_t* err) {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    *err = cudaSuccess;
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        *err = cudaGetSymbolAddress(&p, g_bwd_scratch);
        if (*err == cudaSuccess) g_scratch_ptr[dev] = p;
        else cudaGetLastError();  // the failed lookup must not leak into the next launch check
    }
    return g_scratch_ptr[dev];
}
}  // namespace

extern "C" int lf_laplace_sub_bwd_noalloc(const void* g, const void* q, const void* kT, void* dq, void* dkT,
                                          int64_t bh, int64_t n, int64_t m, int64_t d, int dtype,
                                          lf_stream_t stream) {
    clear_error();
    if ((!dq && bh * n * d > 0) || (!dkT && bh * d * m > 0)) {
        set_error("lf_laplace_sub_bwd_noalloc computes both gradients: dq and dkT must be given");
        return LF_ERR_INVALID;
    }
    const size_t need = lf_laplace_sub_bwd_workspace_size(bh, n, m, d, dtype);
    if (need == 0) return bwd_common(g, q, kT, dq, dkT, bh, n, m, d, dtype, stream);  // no scratch needed
    if (need > kNoAllocScratchBytes) {
        set_error("lf_laplace_sub_bwd_noalloc: this shape needs %zu bytes of scratch, more than its fixed %zu "
                  "(use lf_laplace_sub_bwd_ws or lf_laplace_sub_bwd)", need, kNoAllocScratchBytes);
        return LF_ERR_UNSUPPORTED;
    }
    int rc = check_args(g, q, kT, bh, n, m, d, dtype);
    if (rc) return rc;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDev) {
        set_error("lf_laplace_sub_bwd_noalloc: no usable current device");
        return LF_ERR_CUDA;
    }
    cudaError_t err = cudaSuccess;
    void* scratch = scratch_address(dev, &err);
    if (!scratch) {
        set_error("lf_laplace_sub_bwd_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(err));
        return LF_ERR_CUDA;
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    LF_DISPATCH(dtype, T, return launch_bwd_flat_t<T>(g, q, kT, dq, dkT, bh, n, m, d, scratch,
                                                      kNoAllocScratchBytes, nullptr, st));
    return LF_OK;
}

extern "C" int lf_laplace_sub_bwd_query(const void* g, const void* q, const void* kT, void* dq,
                                        int64_t bh, int64_t n, int64_t m, int64_t d, int dtype,
                                        lf_stream_t stream) {
    clear_error();
    if (!dq && bh * n * d > 0) { set_error("null gradQuery"); return LF_ERR_INVALID; }
    return bwd_common(g, q, kT, dq, nullptr, bh, n, m, d, dtype, stream);
}

extern "C" int lf_laplace_sub_bwd_key(const void* g, const void* q, const void* kT, void* dkT,
                                      int64_t bh, int64_t n, int64_t m, int64_t d, int dtype,
                                      lf_stream_t stream) {
    clear_error();
    if (!dkT && bh * d * m > 0) { set_error("null gradKey"); return LF_ERR_INVALID; }
    return bwd_common(g, q, kT, nullptr, dkT, bh, n, m, d, dtype, stream);
}

extern "C" int lf_laplace_sub_reduce_fwd(const void* q, const void* kT, void* s, int64_t bh,
                                         int64_t n, int64_t m, int64_t d, int dtype,
                                         lf_stream_t stream) {
    clear_error();
    int rc = check_args(q, kT, s, bh, n, m, d, dtype);
    if (rc) return rc;
    int64_t total = bh * n * m;
    if (total == 0) return LF_OK;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (d == 0) {
        if (cudaMemsetAsync(s, 0, (size_t)total * dtype_size(dtype), st) != cudaSuccess) return check_launch("memset");
        return LF_OK;
    }
    int64_t warps_per_block = kThreads / 32;
    int64_t blocks = (total + warps_per_block - 1) / warps_per_block;
    int64_t cap = (int64_t)num_sms() * 16;
    if (blocks > cap) blocks = cap;
    LF_DISPATCH(dtype, T, {
        lsub_reduce_kernel<T><<<(unsigned)blocks, kThreads, 0, st>>>(
            static_cast<const T*>(q), static_cast<const T*>(kT), static_cast<T*>(s), total, (int)n,
            (int)m, (int)d);
        return check_launch("lsub_reduce_kernel");
    });
    return LF_OK;
}
