// Host-resident batches: LaplaceSubtraction forward + both gradients with the
// operands in (pinned) host memory.
//
// The B*H slices are cut into chunks that flow through three CUDA streams —
// copy-in, kernels, copy-out — over a ring of kRing device buffer sets, so
// that the host-to-device copy of chunk i+1, the kernels of chunk i and the
// device-to-host copy of chunk i-1 run at the same time (PCIe is full
// duplex; the kernels of a chunk take a small fraction of its copy time).
// The caller provides the device buffer (lf_laplace_sub_host_buffer_size);
// the library only keeps three streams and a few events per device.
#include <mutex>
#include <vector>

#include "lf_common.cuh"

namespace lfb {
namespace {

constexpr int kRing = 3;
constexpr int kMaxDevP = 64;
constexpr size_t kAlign = 256;

inline size_t up(size_t x) { return (x + kAlign - 1) & ~(kAlign - 1); }

struct Plan {
    int64_t per;         // (b,h) slices of the largest chunk
    std::vector<int64_t> start;  // chunk i covers slices [start[i], start[i+1])
    size_t es;
    size_t q, g, s, dq, ws;  // bytes of each region of one set
    size_t set;              // bytes of one buffer set
    size_t kall;             // K^T (and dK^T) of all slices: copied in once, out once
};

Plan make_plan(int64_t bh, int64_t n, int64_t m, int64_t d, int dtype, int chunks) {
    Plan p{};
    if (chunks < 1) chunks = 1;
    if (chunks > bh) chunks = (int)bh;
    // Equal chunks of `base` slices, except a short first and last chunk
    // (a quarter of base): the pipeline's fill (first copy-in) and drain
    // (last copy-out) run with one direction of PCIe idle, so they are kept
    // short.
    const int64_t base = (bh + chunks - 1) / chunks;
    const int64_t f = base / 4;
    p.start.push_back(0);
    if (f >= 1 && bh > 2 * f + base) {
        const int64_t mid = bh - 2 * f;
        const int64_t nm = (mid + base - 1) / base;
        p.start.push_back(f);
        for (int64_t k = 1; k <= nm; ++k) p.start.push_back(f + (mid * k) / nm);
        p.start.push_back(bh);
    } else {
        for (int64_t a = base; a < bh; a += base) p.start.push_back(a);
        p.start.push_back(bh);
    }
    p.per = base;
    p.es = dtype_size(dtype);
    p.q = up((size_t)p.per * n * d * p.es);
    p.kall = up((size_t)bh * d * m * p.es);
    p.g = up((size_t)p.per * n * m * p.es);
    p.s = p.g;
    p.dq = p.q;
    // workspace need is not monotonic in the slice count (it follows the
    // balanced backward's grid): take the largest over the chunk widths
    p.ws = 0;
    for (size_t i = 0; i + 1 < p.start.size(); ++i) {
        const size_t w = up(lf_laplace_sub_bwd_workspace_size(p.start[i + 1] - p.start[i], n, m, d, dtype));
        if (w > p.ws) p.ws = w;
    }
    p.set = p.q + p.g + p.s + p.dq + p.ws;
    return p;
}

struct DevStreams {
    cudaStream_t in = nullptr, run = nullptr, out = nullptr;
    cudaEvent_t start = nullptr, loaded[kRing] = {}, done[kRing] = {}, freed[kRing] = {};
    cudaError_t err = cudaSuccess;
    std::mutex mu;  // one enqueue at a time per device
};
DevStreams g_dev[kMaxDevP];
std::once_flag g_dev_once[kMaxDevP];

void dev_setup(int dev) {
    DevStreams& s = g_dev[dev];
    auto ok = [&](cudaError_t e) { if (e != cudaSuccess && s.err == cudaSuccess) s.err = e; };
    ok(cudaStreamCreateWithFlags(&s.in, cudaStreamNonBlocking));
    ok(cudaStreamCreateWithFlags(&s.run, cudaStreamNonBlocking));
    ok(cudaStreamCreateWithFlags(&s.out, cudaStreamNonBlocking));
    ok(cudaEventCreateWithFlags(&s.start, cudaEventDisableTiming));
    for (int i = 0; i < kRing; ++i) {
        ok(cudaEventCreateWithFlags(&s.loaded[i], cudaEventDisableTiming));
        ok(cudaEventCreateWithFlags(&s.done[i], cudaEventDisableTiming));
        ok(cudaEventCreateWithFlags(&s.freed[i], cudaEventDisableTiming));
    }
}

#define LF_TRY(call, what)                                                          \
    do {                                                                            \
        cudaError_t e_ = (call);                                                    \
        if (e_ != cudaSuccess) {                                                    \
            set_error("%s: %s", what, cudaGetErrorString(e_));                      \
            return LF_ERR_CUDA;                                                     \
        }                                                                           \
    } while (0)

}  // namespace
}  // namespace lfb

using namespace lfb;

extern "C" size_t lf_laplace_sub_host_buffer_size(int64_t bh, int64_t n, int64_t m, int64_t d, int dtype,
                                                  int chunks) {
    clear_error();
    if (bh <= 0 || n < 0 || m < 0 || d < 0 || dtype_size(dtype) == 0) return 0;
    const Plan p = make_plan(bh, n, m, d, dtype, chunks);
    return p.set * kRing + 2 * p.kall;
}

extern "C" int lf_laplace_sub_fwd_bwd_host(const void* hq, const void* hkT, const void* hg, void* hs, void* hdq,
                                           void* hdkT, int64_t bh, int64_t n, int64_t m, int64_t d, int dtype,
                                           int chunks, void* dbuf, size_t dbuf_bytes, lf_stream_t stream) {
    clear_error();
    if (dtype_size(dtype) == 0) { set_error("unsupported dtype code %d", dtype); return LF_ERR_DTYPE; }
    if (bh < 0 || n < 0 || m < 0 || d < 0) { set_error("negative size"); return LF_ERR_INVALID; }
    if (bh == 0 || n == 0 || m == 0 || d == 0) {
        set_error("lf_laplace_sub_fwd_bwd_host needs bh, n, m, d > 0");
        return LF_ERR_INVALID;
    }
    if (!hq || !hkT || !hg || !hs || !hdq || !hdkT || !dbuf) { set_error("null pointer"); return LF_ERR_INVALID; }
    if (reinterpret_cast<uintptr_t>(dbuf) % kAlign) {
        set_error("lf_laplace_sub_fwd_bwd_host: device buffer must be %zu-byte aligned", kAlign);
        return LF_ERR_INVALID;
    }
    const Plan p = make_plan(bh, n, m, d, dtype, chunks);
    if (dbuf_bytes < p.set * kRing + 2 * p.kall) {
        set_error("lf_laplace_sub_fwd_bwd_host: device buffer of %zu bytes, %zu needed", dbuf_bytes,
                  p.set * kRing + 2 * p.kall);
        return LF_ERR_INVALID;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevP) {
        set_error("lf_laplace_sub_fwd_bwd_host: no usable current device");
        return LF_ERR_CUDA;
    }
    std::call_once(g_dev_once[dev], dev_setup, dev);
    DevStreams& S = g_dev[dev];
    if (S.err != cudaSuccess) {
        set_error("lf_laplace_sub_fwd_bwd_host: stream/event creation failed: %s", cudaGetErrorString(S.err));
        return LF_ERR_CUDA;
    }
    std::lock_guard<std::mutex> lock(S.mu);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const size_t es = p.es;
    const char* Hq = static_cast<const char*>(hq);
    const char* Hk = static_cast<const char*>(hkT);
    const char* Hg = static_cast<const char*>(hg);
    char* Hs = static_cast<char*>(hs);
    char* Hdq = static_cast<char*>(hdq);
    char* Hdk = static_cast<char*>(hdkT);
    char* base = static_cast<char*>(dbuf);

    LF_TRY(cudaEventRecord(S.start, st), "cudaEventRecord");
    LF_TRY(cudaStreamWaitEvent(S.in, S.start, 0), "cudaStreamWaitEvent");
    LF_TRY(cudaStreamWaitEvent(S.run, S.start, 0), "cudaStreamWaitEvent");
    LF_TRY(cudaStreamWaitEvent(S.out, S.start, 0), "cudaStreamWaitEvent");
    const int64_t nchunks = (int64_t)p.start.size() - 1;
    // K^T is small (d x m per slice): one copy in before the chunks and one
    // copy of dK^T out after them, instead of two small copies per chunk
    // (each costs a fixed ~10 us of the copy engines' time).
    char* kall = base + (size_t)kRing * p.set;
    char* dkall = kall + p.kall;
    LF_TRY(cudaMemcpyAsync(kall, Hk, (size_t)bh * d * m * es, cudaMemcpyHostToDevice, S.in), "copy-in");
    for (int64_t i = 0; i < nchunks; ++i) {
        const int r = (int)(i % kRing);
        const int64_t a = p.start[i];
        const int64_t w = p.start[i + 1] - a;
        char* b = base + (size_t)r * p.set;
        char* dq_in = b;
        char* dg_in = dq_in + p.q;
        char* ds_out = dg_in + p.g;
        char* ddq_out = ds_out + p.s;
        char* dws = ddq_out + p.dq;
        char* dk_in = kall + (size_t)a * d * m * es;
        char* ddk_out = dkall + (size_t)a * d * m * es;
        const size_t bq = (size_t)w * n * d * es, bg = (size_t)w * n * m * es;
        // copy-in; the set is free once the copy-out kRing chunks back is done
        if (i >= kRing) LF_TRY(cudaStreamWaitEvent(S.in, S.freed[r], 0), "cudaStreamWaitEvent");
        LF_TRY(cudaMemcpyAsync(dq_in, Hq + (size_t)a * n * d * es, bq, cudaMemcpyHostToDevice, S.in), "copy-in");
        LF_TRY(cudaMemcpyAsync(dg_in, Hg + (size_t)a * n * m * es, bg, cudaMemcpyHostToDevice, S.in), "copy-in");
        LF_TRY(cudaEventRecord(S.loaded[r], S.in), "cudaEventRecord");
        // kernels
        LF_TRY(cudaStreamWaitEvent(S.run, S.loaded[r], 0), "cudaStreamWaitEvent");
        lf_stream_t rs = reinterpret_cast<lf_stream_t>(S.run);
        int rc = lf_laplace_sub_fwd(dq_in, dk_in, ds_out, w, n, m, d, dtype, rs);
        if (rc) return rc;
        rc = p.ws ? lf_laplace_sub_bwd_ws(dg_in, dq_in, dk_in, ddq_out, ddk_out, w, n, m, d, dtype, dws, p.ws, rs)
                  : lf_laplace_sub_bwd(dg_in, dq_in, dk_in, ddq_out, ddk_out, w, n, m, d, dtype, rs);
        if (rc) return rc;
        LF_TRY(cudaEventRecord(S.done[r], S.run), "cudaEventRecord");
        // copy-out
        LF_TRY(cudaStreamWaitEvent(S.out, S.done[r], 0), "cudaStreamWaitEvent");
        LF_TRY(cudaMemcpyAsync(Hs + (size_t)a * n * m * es, ds_out, bg, cudaMemcpyDeviceToHost, S.out), "copy-out");
        LF_TRY(cudaMemcpyAsync(Hdq + (size_t)a * n * d * es, ddq_out, bq, cudaMemcpyDeviceToHost, S.out), "copy-out");
        LF_TRY(cudaEventRecord(S.freed[r], S.out), "cudaEventRecord");
    }
    // dK^T of every slice (the kernels run in stream order: the last chunk's
    // completion covers all), then the caller's stream continues after the
    // last copy-out
    LF_TRY(cudaMemcpyAsync(Hdk, dkall, (size_t)bh * d * m * es, cudaMemcpyDeviceToHost, S.out), "copy-out");
    LF_TRY(cudaEventRecord(S.freed[(nchunks - 1) % kRing], S.out), "cudaEventRecord");
    LF_TRY(cudaStreamWaitEvent(st, S.freed[(nchunks - 1) % kRing], 0), "cudaStreamWaitEvent");
    return LF_OK;
}
