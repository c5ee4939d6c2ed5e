// Library-wide C ABI pieces: version, thread-local error strings, device
// attribute cache.
#include <stdarg.h>
#include <stdio.h>

#include <mutex>

#include "fc_common.cuh"

#define FC_VERSION_STRING "flashcodec_b200 0.1.0 sm_100a"

namespace fc {

static thread_local char g_err[512] = {0};

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

void clear_error() { g_err[0] = 0; }

int check_launch(const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error("%s: CUDA error %d (%s)", what, (int)e, cudaGetErrorString(e));
        return FC_ECUDA;
    }
    return FC_OK;
}

int num_sms() {
    static std::mutex mu;
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    std::lock_guard<std::mutex> lock(mu);
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

}  // namespace fc

extern "C" const char *fc_version(void) { return FC_VERSION_STRING; }

extern "C" const char *fc_last_error_string(void) { return fc::g_err; }
