/*
 * laplacian_b200.h — C ABI of the B200 (sm_100a) LaplacianFormer operators.
 *
 * Plain pointers, sizes and a CUDA stream; no framework types.  Every tensor
 * is dense, row-major and lives in device memory of the current CUDA device.
 * Calls are asynchronous on `stream` (0 = legacy default stream), never
 * allocate memory and never synchronise.  Each entry point returns LF_OK or
 * one of the LF_ERR_* codes; lf_last_error() returns a message for the most
 * recent failure on the calling host thread.
 *
 * Layouts follow the reference operators (BirdWithDreams/LaplacianFormer):
 *   query  Q   [bh, n, d]      (the reference's [B,H,N,D], bh = B*H)
 *   key    KT  [bh, d, m]      (the reference's [B,H,D,M]: landmarks transposed,
 *                               src/LaplaceSubtraction_cuda.cu:25-27, :62)
 *   output S   [bh, n, m]
 *   matrices   [batch, n, n]   (the reference's [B,H,N,N], batch = B*H)
 *
 * The reference binds its operators with pybind11 (src/wrapper.cpp:73-98);
 * each entry point below names the reference function it replaces.
 */
#ifndef LAPLACIAN_B200_H
#define LAPLACIAN_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define LF_API __attribute__((visibility("default")))
#else
#define LF_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* lf_stream_t; /* == cudaStream_t */

/* Element types (all operands of one call share it). */
enum lf_dtype {
    LF_F32 = 0,
    LF_F64 = 1,
    LF_F16 = 2,
    LF_BF16 = 3
};

/* Status codes. */
enum lf_status {
    LF_OK = 0,
    LF_ERR_INVALID = 1,      /* bad pointer, size or stride                  */
    LF_ERR_DTYPE = 2,        /* element type not supported by this operator  */
    LF_ERR_UNSUPPORTED = 3,  /* size outside the supported range             */
    LF_ERR_CUDA = 4,         /* a CUDA runtime call or launch failed         */
    LF_ERR_TIMEOUT = 5       /* a device-side bounded wait expired           */
};

/* Remote destinations of the peer (NVLink) entry points: a node's other
   GPUs, and the bytes of a peer-buffer handle (a CUDA IPC handle). */
#define LF_MAX_PEERS 8
#define LF_PEER_HANDLE_BYTES 64

/* NewtonInverse initialisation modes. */
enum lf_ns_init {
    /* P = A + reg*I, V0 = 1.8 / (max_i sum_j P_ij)^2 * P
       (src/NewtonInverse_cuda_kernel.cu:82-120, :169, :176-178). */
    LF_NS_INIT_REFERENCE = 0,
    /* P = A + reg*I, X0 = P^T / (||P||_1 ||P||_inf). */
    LF_NS_INIT_SCALED_TRANSPOSE = 1
};

/* NewtonInverse arithmetic for fp32 / fp16 / bf16 inputs. */
enum lf_ns_precision {
    /* Every product on tcgen05 tensor cores as hi*hi + hi*lo + lo*hi fp16
       parts with fp32 accumulation (about 22 significant bits). */
    LF_NS_PREC_SPLIT3 = 0,
    /* Single fp16 product for all but the last two iterations, split
       products for the last two (Newton–Schulz corrects earlier rounding). */
    LF_NS_PREC_MIXED = 1,
    /* CUDA-core fp32 FMA for every product (no tensor cores). */
    LF_NS_PREC_FP32_SIMT = 2
};

/* ---------------------------------------------------------------------- */
/* Library information                                                     */
/* ---------------------------------------------------------------------- */

/* Message describing the last failure on this host thread ("" if none). */
LF_API const char* lf_last_error(void);
/* CUDART_VERSION the library was built with.
   Replaces laplace::get_cudart_version (src/cuda_version.cu:7-26). */
LF_API int lf_cudart_version(void);
/* Library version as major*10000 + minor*100 + patch. */
LF_API int lf_version(void);

/* ---------------------------------------------------------------------- */
/* LaplaceSubtraction                                                      */
/* ---------------------------------------------------------------------- */

/* S[b,i,j] = sum_c |Q[b,i,c] - KT[b,c,j]|.  dtype: F32, F64, F16, BF16.
   Replaces laplace::LaplaceSubtraction_forward_cuda
   (src/LaplaceSubtraction_cuda.cu:55-67 -> src/LaplaceSubtraction_cuda_kernel.cu:455-485). */
LF_API int lf_laplace_sub_fwd(const void* q, const void* kT, void* s,
                       int64_t bh, int64_t n, int64_t m, int64_t d,
                       int dtype, lf_stream_t stream);

/* lf_laplace_sub_fwd for fp16 storage with packed half2 arithmetic: the
   differences and 16-channel partial sums are fp16 pairs, the partials are
   added in fp32.  Opt-in and not bit-identical: within ~1e-3 relative of the
   fp32 channel sum (the half-precision tolerance of the path is 1e-2).
   fp16 only (LF_ERR_DTYPE otherwise), d <= 64.  No counterpart in the
   reference (its half path converts to fp32, LaplaceSubtraction_cuda_kernel.cu:471). */
LF_API int lf_laplace_sub_fwd_packed(const void* q, const void* kT, void* s,
                       int64_t bh, int64_t n, int64_t m, int64_t d,
                       int dtype, lf_stream_t stream);

/* Laplacian kernel matrix Kmat[b,i,j] = exp(scale * S[b,i,j]) with S as in
   lf_laplace_sub_fwd (the same bit-exact channel sums), the exponential
   applied in the accumulation type before the one rounding to the storage
   type; the attention block uses scale = -1/sigma.  S is never written.
   Gradients: dS = scale * Kmat * dKmat, then lf_laplace_sub_bwd.  No
   counterpart in the reference (its attention applies exp as a separate
   PyTorch op on the stored S). */
LF_API int lf_laplace_kernel_fwd(const void* q, const void* kT, void* kmat,
                          int64_t bh, int64_t n, int64_t m, int64_t d,
                          int dtype, double scale, lf_stream_t stream);

/* Gradients of Kmat = exp(scale * S) (lf_laplace_kernel_fwd) from the
   upstream gradient GK = dKmat: dS = scale * Kmat * GK is formed inside the
   backward kernels while they stage their gradient tile (in the accumulation
   type), then dQ and dKT follow as in lf_laplace_sub_bwd; dS is never
   written to or read from memory.  kmat is the forward's output.  Either of
   dq, dkT may be NULL.  `workspace` (NULL, or at least
   lf_laplace_sub_bwd_workspace_size bytes, 16-byte aligned) selects the
   balanced launch of lf_laplace_sub_bwd_ws when both gradients are asked
   for.  No counterpart in the reference (its attention forms dS with
   separate PyTorch ops before LaplaceSubtraction_backward_query/_key). */
LF_API int lf_laplace_kernel_bwd(const void* gk, const void* kmat, const void* q, const void* kT,
                          void* dq, void* dkT,
                          int64_t bh, int64_t n, int64_t m, int64_t d,
                          int dtype, double scale, void* workspace, size_t workspace_bytes,
                          lf_stream_t stream);

/* dQ[b,i,c] = sum_j G[b,i,j] * sign(Q[b,i,c] - KT[b,c,j]), sign(0) = 0.
   Replaces laplace::LaplaceSubtraction_backward_query_cuda
   (src/LaplaceSubtraction_cuda.cu:69-84 -> src/LaplaceSubtraction_cuda_kernel.cu:487-547). */
LF_API int lf_laplace_sub_bwd_query(const void* g, const void* q, const void* kT, void* dq,
                             int64_t bh, int64_t n, int64_t m, int64_t d,
                             int dtype, lf_stream_t stream);

/* dKT[b,c,j] = -sum_i G[b,i,j] * sign(Q[b,i,c] - KT[b,c,j]).
   Replaces laplace::LaplaceSubtraction_backward_key_cuda
   (src/LaplaceSubtraction_cuda.cu:86-101 -> src/LaplaceSubtraction_cuda_kernel.cu:549-609). */
LF_API int lf_laplace_sub_bwd_key(const void* g, const void* q, const void* kT, void* dkT,
                           int64_t bh, int64_t n, int64_t m, int64_t d,
                           int dtype, lf_stream_t stream);

/* Both gradients from one pass over G; either output may be NULL.  Has no
   single counterpart in the reference, which reads G once per gradient
   (src/LaplaceSubtraction_cuda_kernel.cu:487-609). */
LF_API int lf_laplace_sub_bwd(const void* g, const void* q, const void* kT,
                       void* dq, void* dkT,
                       int64_t bh, int64_t n, int64_t m, int64_t d,
                       int dtype, lf_stream_t stream);

/* Device workspace bytes that lf_laplace_sub_bwd_ws takes for this shape on
   the current device (it depends on the SM count); 0 when the shape runs
   without workspace (d > 32, m > 64 or F64).  No counterpart in the
   reference. */
LF_API size_t lf_laplace_sub_bwd_workspace_size(int64_t bh, int64_t n, int64_t m, int64_t d, int dtype);

/* lf_laplace_sub_bwd (both gradients) with the row chunks of all (b,h)
   spread evenly over every SM: each CTA takes a contiguous run of 64-row
   chunks that may cross (b,h) boundaries, and the dKT partials of the (b,h)
   shared by several CTAs meet in `workspace` (16-byte aligned device memory
   of at least lf_laplace_sub_bwd_workspace_size bytes; nothing in it needs
   to be initialised), summed by a second kernel in a fixed order.  When the
   size query gives 0, or dq or dkT is NULL, this is lf_laplace_sub_bwd and
   the workspace is not touched.  Concurrent calls need distinct workspaces.
   No counterpart in the reference, which splits rows with atomicAdd into a
   zeroed output (src/LaplaceSubtraction_cuda_kernel.cu:568-580). */
LF_API int lf_laplace_sub_bwd_ws(const void* g, const void* q, const void* kT,
                          void* dq, void* dkT,
                          int64_t bh, int64_t n, int64_t m, int64_t d,
                          int dtype, void* workspace, size_t workspace_bytes,
                          lf_stream_t stream);

/* Size of the fixed device scratch of lf_laplace_sub_bwd_noalloc. */
#define LF_BWD_NOALLOC_SCRATCH_BYTES (2u << 20)

/* lf_laplace_sub_bwd_ws for callers that cannot allocate device memory: code
   running where cudaMalloc is not allowed or not wanted (inside a custom
   allocator or memory-pool callback, a host that has handed all device memory
   to its own pool, or a real-time loop that must not synchronise, which
   cudaMalloc/cudaFree can do).  Its workspace is a fixed 2 MiB array
   (LF_BWD_NOALLOC_SCRATCH_BYTES) compiled into the library, which every GPU
   that loads the library holds until the process exits; nothing is allocated
   per call.  Both dq and dkT are required.  Shapes whose
   lf_laplace_sub_bwd_workspace_size exceeds 2 MiB are rejected with
   LF_ERR_UNSUPPORTED; shapes with size 0 run lf_laplace_sub_bwd.  The first
   call on a device looks up the array's device address (cudaGetSymbolAddress)
   with that device current; make that first call before any stream capture
   (a failed lookup is reported as LF_ERR_CUDA and retried by the next call).
   All calls share the one array and each overwrites what it reads (nothing
   needs to start at zero), so calls that can overlap on the GPU (different
   streams or host threads) race: serialise them.  No counterpart in the
   reference. */
LF_API int lf_laplace_sub_bwd_noalloc(const void* g, const void* q, const void* kT,
                               void* dq, void* dkT,
                               int64_t bh, int64_t n, int64_t m, int64_t d,
                               int dtype, lf_stream_t stream);

/* Device buffer bytes lf_laplace_sub_fwd_bwd_host needs for this shape and
   chunk count (three rotating sets of per-chunk operands, results and
   backward workspace).  No counterpart in the reference. */
LF_API size_t lf_laplace_sub_host_buffer_size(int64_t bh, int64_t n, int64_t m, int64_t d, int dtype,
                                       int chunks);

/* Forward S and both gradients dQ, dKT for operands in HOST memory (pinned,
   for the copies to overlap): q, kT, g are read and s, dq, dkT written in
   host memory.  The bh slices are cut into `chunks` pieces that stream
   through host-to-device copies, the kernels and device-to-host copies on
   three library-owned streams, so both PCIe directions and the kernels
   overlap.  `dbuf` is a 256-byte aligned device buffer of at least
   lf_laplace_sub_host_buffer_size bytes.  Asynchronous: `stream` waits for
   the last copy-out (synchronise it before reading the host results).  The
   first call on a device creates its streams and events.  No counterpart in
   the reference, whose operators take device tensors only. */
LF_API int lf_laplace_sub_fwd_bwd_host(const void* q, const void* kT, const void* g,
                                void* s, void* dq, void* dkT,
                                int64_t bh, int64_t n, int64_t m, int64_t d, int dtype,
                                int chunks, void* dbuf, size_t dbuf_bytes, lf_stream_t stream);

/* Legacy forward with the reference's per-output tree reduction in the
   storage type, including its behaviour for d that is not a power of two.
   Replaces laplace::LaplaceSubtraction_reduce_forward_cuda
   (src/LaplaceSubtraction_cuda.cu:103-116 -> src/LaplaceSubtraction_cuda_kernel.cu:611-647). */
LF_API int lf_laplace_sub_reduce_fwd(const void* q, const void* kT, void* s,
                              int64_t bh, int64_t n, int64_t m, int64_t d,
                              int dtype, lf_stream_t stream);

/* ---------------------------------------------------------------------- */
/* NewtonInverse                                                           */
/* ---------------------------------------------------------------------- */

/* 1 if n is supported by lf_newton_inverse_fwd / _bwd, else 0.
   Replaces laplace::NewtonInverse_supports (src/NewtonInverse_cuda_kernel.cu:753-762). */
LF_API int lf_newton_inverse_supported(int64_t n);

/* Reference semantics: P = A + 0.01 I, V0 = alpha P, `iters` steps of
   V <- 2V - V P V.  dtype: F32, F64, F16, BF16.
   Replaces laplace::NewtonInverse_forward_cuda (src/NewtonInverse_cuda_kernel.cu:764-794). */
LF_API int lf_newton_inverse_fwd(const void* a, void* x, int64_t batch, int64_t n, int iters,
                          int dtype, lf_stream_t stream);

/* Extended forward: init mode (lf_ns_init), diagonal regulariser `reg` and
   arithmetic (lf_ns_precision).  lf_newton_inverse_fwd(...) is
   lf_newton_inverse_fwd_ex(..., LF_NS_INIT_REFERENCE, 0.01, LF_NS_PREC_SPLIT3, ...).
   No counterpart in the reference, whose constants are hard-coded
   (src/NewtonInverse_cuda_kernel.cu:116, :169). */
LF_API int lf_newton_inverse_fwd_ex(const void* a, void* x, int64_t batch, int64_t n, int iters,
                             int dtype, int init_mode, double reg, int precision,
                             lf_stream_t stream);

/* Newton–Schulz inverse of the landmark kernel matrix built in the same
   kernel: A_b = exp(scale * S_b), S_b[i][j] = sum_k |L_b[i][k] - L_b[j][k]|
   (bit-identical to lf_laplace_kernel_fwd(L, L^T, scale)), then
   lf_newton_inverse_fwd_ex(A, ...) on the tensor cores — A never goes to
   global memory.  L is fp32 [batch, n, d], X fp32 [batch, n, n]; n <= 128,
   d <= 128, precision LF_NS_PREC_SPLIT3 or LF_NS_PREC_MIXED.  No counterpart
   in the reference, where A is three separate PyTorch/CUDA steps. */
LF_API int lf_laplace_newton_inverse_fwd(const void* lmk, void* x, int64_t batch, int64_t n, int64_t d,
                                  double scale, int iters, int init_mode, double reg, int precision,
                                  lf_stream_t stream);

/* dA = -(V^T G V^T) for the inverse V and upstream gradient G.
   Replaces laplace::NewtonInverse_backward_cuda (src/NewtonInverse_cuda_kernel.cu:796-833). */
LF_API int lf_newton_inverse_bwd(const void* g, const void* v, void* da,
                          int64_t batch, int64_t n, int dtype, lf_stream_t stream);

/* res[b] = ||(A_b + reg I) X_b - I||_F in fp32 (fp64 for F64 input), the
   per-matrix residual the batched benchmark reports.  No counterpart in the
   reference. */
LF_API int lf_newton_inverse_residual(const void* a, const void* x, void* res,
                               int64_t batch, int64_t n, double reg,
                               int dtype, lf_stream_t stream);

/* Synchronises the current device and returns the status word that kernels
   set when a bounded device-side wait expires (LF_OK if none); clear != 0
   resets it.  No counterpart in the reference, which can only printf launch
   errors (src/NewtonInverse_cuda_kernel.cu:790-793). */
LF_API int lf_device_status(int clear);

/* Launches a one-block kernel that waits on a barrier nothing completes; the
   bounded wait gives up after timeout_ms (1..10000) and records LF_ERR_TIMEOUT
   in the device status word (read it with lf_device_status).  Exercises the
   error path the tensor-core kernels take instead of hanging.  No
   counterpart in the reference. */
LF_API int lf_selftest_bounded_wait(int timeout_ms, lf_stream_t stream);

/* ---------------------------------------------------------------------------
   Gather of a (b,h)-sharded run over NVLink peer memory.  The reference has no
   multi-GPU code; its callers shard B*H over ranks and all-gather dQ, dK^T
   and X with a collective afterwards.  These entry points let the producing
   kernels write every rank's copy directly, one process per GPU.
   ------------------------------------------------------------------------- */

/* cudaMalloc(bytes), zeroed, and its IPC handle (LF_PEER_HANDLE_BYTES bytes
   written to `handle`) for the other ranks to map with lf_peer_open.
   Synchronous; free with lf_peer_free. */
LF_API int lf_peer_alloc(size_t bytes, void** ptr, void* handle);

/* Maps another process's lf_peer_alloc buffer (same node) into this device's
   address space; unmap with lf_peer_close.  Synchronous. */
LF_API int lf_peer_open(const void* handle, void** ptr);
LF_API int lf_peer_close(void* ptr);
LF_API int lf_peer_free(void* ptr);

/* Copies `bytes` from local device memory `src` to each of the `ndst`
   (<= LF_MAX_PEERS) destinations (local or peer device pointers). */
LF_API int lf_peer_put(const void* src, size_t bytes, void* const* dsts, int ndst, lf_stream_t stream);

/* Stream-ordered barrier of `world` ranks (<= LF_MAX_PEERS + 1):
   flags[r] is rank r's uint32 flag array of `world` entries (an lf_peer_alloc
   buffer, mapped here with lf_peer_open; flags[rank] is this rank's own).
   Writes `epoch` into flags[r][rank] of every peer r with a system-scope
   release after all earlier work on the stream, then waits until
   flags[rank][r] has reached `epoch` for every peer r (so every peer's
   earlier stores into this GPU are visible to later work on the stream).
   Epochs must increase by one per call.  A wait longer than timeout_ms
   (1..60000) gives up and records LF_ERR_TIMEOUT in the device status word
   (lf_device_status). */
LF_API int lf_peer_barrier(uint32_t* const* flags, int world, int rank, uint32_t epoch, int timeout_ms,
                           lf_stream_t stream);

/* lf_laplace_sub_bwd_ws that also stores dQ at the same element offsets into
   each of the `npeer` (<= LF_MAX_PEERS) buffers dq_peers[i] (peer device
   pointers from lf_peer_open, already offset to this rank's slice), so the
   all-gather of dQ overlaps the backward.  Shapes the balanced wide kernel
   (d <= 64, 128 < m <= 256) runs store from inside the kernel; other shapes
   run lf_laplace_sub_bwd_ws and then lf_peer_put.  dK^T is written locally
   only (push it with lf_peer_put).  Finish with lf_peer_barrier before a
   peer reads its buffer. */
LF_API int lf_laplace_sub_bwd_peers(const void* g, const void* q, const void* kT,
                                    void* dq, void* dkT, void* const* dq_peers, int npeer,
                                    int64_t bh, int64_t n, int64_t m, int64_t d, int dtype,
                                    void* workspace, size_t workspace_bytes, lf_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* LAPLACIAN_B200_H */
