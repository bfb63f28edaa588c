// Peer memory for the sharded backward's all-gather over NVLink.
//
// The reference has no multi-GPU code; its callers all-gather the outputs of
// a (b,h)-sharded run with a collective after the compute.  Here the gather
// is folded into the producing kernels: every rank maps the other ranks'
// gather buffers (CUDA IPC, one cudaMalloc per buffer so a handle names the
// whole allocation), and the balanced wide backward stores each dQ tile into
// the local buffer and into every peer's buffer at the same offset, so the
// NVLink writes overlap the arithmetic tile by tile.  Small outputs (dK^T,
// the inverse X) are pushed by lf_peer_put.  lf_peer_barrier then publishes
// an epoch to every peer's flag array with a system-scope release and waits,
// with a time limit, until every peer's epoch has arrived; an expired wait
// records LF_ERR_TIMEOUT in the device status word instead of hanging.
#include "lf_common.cuh"

namespace lfb {

__device__ int g_peer_status = 0;

// Host side of the status word (merged into lf_device_status).
int peer_status(bool clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_peer_status, sizeof(int)) != cudaSuccess) return LF_ERR_CUDA;
    if (clear && v) {
        int z = 0;
        if (cudaMemcpyToSymbol(g_peer_status, &z, sizeof(int)) != cudaSuccess) return LF_ERR_CUDA;
    }
    return v;
}

namespace {

struct PeerDst {
    void* p[LF_MAX_PEERS];
    int n;
};

struct PeerFlags {
    uint32_t* flag[LF_MAX_PEERS + 1];  // flag array of each rank (this rank's included)
    int world, rank;
};

__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// One warp: lane r != rank signals rank r, then waits for rank r's signal.
__global__ void peer_barrier_kernel(PeerFlags f, uint32_t epoch, uint64_t limit_ns) {
    const int r = threadIdx.x;
    const bool peer = r < f.world && r != f.rank;
    if (peer) {
        __threadfence_system();
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f.flag[r] + f.rank), "r"(epoch) : "memory");
        const uint32_t* mine = f.flag[f.rank] + r;
        const uint64_t t0 = now_ns();
        for (;;) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
            if ((int32_t)(v - epoch) >= 0) break;
            if (now_ns() - t0 > limit_ns) {
                atomicCAS(&g_peer_status, 0, (int)LF_ERR_TIMEOUT);
                break;
            }
            __nanosleep(256);
        }
    }
    __syncwarp();
    __threadfence_system();
}

// dst[i][e] = src[e] for every destination, 16 bytes per thread and step.
__global__ void peer_put_kernel(const uint4* __restrict__ src, size_t n16, PeerDst dst) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < n16; e += stride) {
        const uint4 v = src[e];
#pragma unroll
        for (int i = 0; i < LF_MAX_PEERS; ++i)
            if (i < dst.n) static_cast<uint4*>(dst.p[i])[e] = v;
    }
}

__global__ void peer_put_bytes_kernel(const unsigned char* __restrict__ src, size_t n, PeerDst dst) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += stride) {
        const unsigned char v = src[e];
#pragma unroll
        for (int i = 0; i < LF_MAX_PEERS; ++i)
            if (i < dst.n) static_cast<unsigned char*>(dst.p[i])[e] = v;
    }
}

}  // namespace
}  // namespace lfb

using namespace lfb;

extern "C" int lf_peer_alloc(size_t bytes, void** ptr, void* handle) {
    clear_error();
    if (!ptr || !handle || bytes == 0) { set_error("lf_peer_alloc: null argument or zero size"); return LF_ERR_INVALID; }
    *ptr = nullptr;
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return check_launch("lf_peer_alloc: cudaMalloc");
    if (cudaMemset(p, 0, bytes) != cudaSuccess) { cudaFree(p); return check_launch("lf_peer_alloc: cudaMemset"); }
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
        cudaFree(p);
        return check_launch("lf_peer_alloc: cudaIpcGetMemHandle");
    }
    static_assert(sizeof(h) == LF_PEER_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &h, sizeof(h));
    *ptr = p;
    return LF_OK;
}

extern "C" int lf_peer_open(const void* handle, void** ptr) {
    clear_error();
    if (!ptr || !handle) { set_error("lf_peer_open: null argument"); return LF_ERR_INVALID; }
    *ptr = nullptr;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
        return check_launch("lf_peer_open: cudaIpcOpenMemHandle");
    *ptr = p;
    return LF_OK;
}

extern "C" int lf_peer_close(void* ptr) {
    clear_error();
    if (!ptr) return LF_OK;
    if (cudaIpcCloseMemHandle(ptr) != cudaSuccess) return check_launch("lf_peer_close");
    return LF_OK;
}

extern "C" int lf_peer_free(void* ptr) {
    clear_error();
    if (!ptr) return LF_OK;
    if (cudaFree(ptr) != cudaSuccess) return check_launch("lf_peer_free");
    return LF_OK;
}

extern "C" int lf_peer_put(const void* src, size_t bytes, void* const* dsts, int ndst, lf_stream_t stream) {
    clear_error();
    if (ndst < 0 || ndst > LF_MAX_PEERS) { set_error("lf_peer_put: %d destinations (at most %d)", ndst, LF_MAX_PEERS); return LF_ERR_INVALID; }
    if (bytes == 0 || ndst == 0) return LF_OK;
    if (!src || !dsts) { set_error("lf_peer_put: null pointer"); return LF_ERR_INVALID; }
    PeerDst d = {};
    d.n = ndst;
    bool a16 = aligned(src, 16) && bytes % 16 == 0;
    for (int i = 0; i < ndst; ++i) {
        if (!dsts[i]) { set_error("lf_peer_put: null destination %d", i); return LF_ERR_INVALID; }
        d.p[i] = dsts[i];
        a16 = a16 && aligned(dsts[i], 16);
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    // A few CTAs per SM keep enough 16-byte stores in flight to fill the
    // links while leaving most of the GPU to a concurrent kernel.
    const size_t units = a16 ? bytes / 16 : bytes;
    const int blocks = (int)((units + 255) / 256 < (size_t)(2 * num_sms()) ? (units + 255) / 256 : (size_t)(2 * num_sms()));
    if (a16) peer_put_kernel<<<blocks, 256, 0, st>>>(static_cast<const uint4*>(src), units, d);
    else peer_put_bytes_kernel<<<blocks, 256, 0, st>>>(static_cast<const unsigned char*>(src), units, d);
    return check_launch("peer_put_kernel");
}

extern "C" int lf_peer_barrier(uint32_t* const* flags, int world, int rank, uint32_t epoch, int timeout_ms,
                               lf_stream_t stream) {
    clear_error();
    if (world < 1 || world > LF_MAX_PEERS + 1 || rank < 0 || rank >= world) {
        set_error("lf_peer_barrier: rank %d of %d (at most %d ranks)", rank, world, LF_MAX_PEERS + 1);
        return LF_ERR_INVALID;
    }
    if (timeout_ms < 1 || timeout_ms > 60000) { set_error("lf_peer_barrier: timeout_ms must be in [1, 60000]"); return LF_ERR_INVALID; }
    if (world == 1) return LF_OK;
    if (!flags) { set_error("lf_peer_barrier: null flag table"); return LF_ERR_INVALID; }
    PeerFlags f = {};
    f.world = world;
    f.rank = rank;
    for (int r = 0; r < world; ++r) {
        if (!flags[r] || !aligned(flags[r], 4)) { set_error("lf_peer_barrier: bad flag array of rank %d", r); return LF_ERR_INVALID; }
        f.flag[r] = flags[r];
    }
    peer_barrier_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(f, epoch, (uint64_t)timeout_ms * 1000000ull);
    return check_launch("peer_barrier_kernel");
}
