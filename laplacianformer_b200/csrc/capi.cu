// Library-wide state of the C ABI: per-thread error messages and cached
// device properties.
#include <stdarg.h>

#include <mutex>

#include "lf_common.cuh"

namespace lfb {

static thread_local char g_err[512] = {0};

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

void clear_error() { g_err[0] = 0; }

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error("%s: %s", what, cudaGetErrorString(e));
        return LF_ERR_CUDA;
    }
    return LF_OK;
}

namespace {
constexpr int kMaxDev = 64;
int g_sms[kMaxDev];
int g_smem[kMaxDev];
std::once_flag g_once[kMaxDev];

void query(int dev) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    g_sms[dev] = v > 0 ? v : 148;
    v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    g_smem[dev] = v > 0 ? v : 48 * 1024;
}

int current_dev() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) dev = 0;
    return dev;
}
}  // namespace

int num_sms() {
    int dev = current_dev();
    std::call_once(g_once[dev], query, dev);
    return g_sms[dev];
}

int max_optin_smem() {
    int dev = current_dev();
    std::call_once(g_once[dev], query, dev);
    return g_smem[dev];
}

}  // namespace lfb

extern "C" const char* lf_last_error(void) { return lfb::g_err; }
extern "C" int lf_cudart_version(void) { return CUDART_VERSION; }
extern "C" int lf_version(void) { return 100; }
