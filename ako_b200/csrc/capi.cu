// Status and error reporting of the C ABI (declared in include/ako_b200.h).
#include <atomic>
#include <cstdarg>
#include <cstdio>

#include "host.hpp"

namespace ako_b200 {

namespace {
thread_local char g_last_error[512] = {0};
constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {0};
std::atomic<int> g_pdl{1};
}  // namespace

bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed) != 0; }

int set_error(int status, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return status;
}

int clear_error() {
    g_last_error[0] = '\0';
    return AKO_B200_OK;
}

int check_launch(const char* kernel) {
    const cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) {
        return set_error(AKO_B200_ERR_CUDA, "%s: launch failed: %s (%s)", kernel,
                         cudaGetErrorString(err), cudaGetErrorName(err));
    }
    return AKO_B200_OK;
}

int sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
    if (g_sm_count[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        g_sm_count[dev] = n;
    }
    return g_sm_count[dev];
}

}  // namespace ako_b200

extern "C" {

int ako_b200_abi_version(void) { return AKO_B200_ABI_VERSION; }

const char* ako_b200_status_string(int status) {
    switch (status) {
        case AKO_B200_OK: return "AKO_B200_OK";
        case AKO_B200_ERR_INVALID_ARGUMENT: return "AKO_B200_ERR_INVALID_ARGUMENT";
        case AKO_B200_ERR_UNSUPPORTED_DTYPE: return "AKO_B200_ERR_UNSUPPORTED_DTYPE";
        case AKO_B200_ERR_CUDA: return "AKO_B200_ERR_CUDA";
        default: return "AKO_B200_ERR_UNKNOWN";
    }
}

const char* ako_b200_last_error(void) { return ako_b200::g_last_error; }

int ako_b200_set_pdl(int enable) { return ako_b200::g_pdl.exchange(enable ? 1 : 0); }

}  // extern "C"
