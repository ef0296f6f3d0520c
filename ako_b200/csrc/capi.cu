// Status and error reporting of the C ABI (declared in include/ako_b200.h),
// and the host-mapped status word of the persistent kernels.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "host.hpp"

namespace ako_b200 {

namespace {
thread_local char g_last_error[512] = {0};
constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {0};
#ifdef AKO_B200_MEASUREMENT
std::atomic<int> g_pdl{1};
#endif
std::mutex g_status_mutex;
std::atomic<int*> g_status_word{nullptr};
}  // namespace

#ifdef AKO_B200_MEASUREMENT
bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed) != 0; }
#else
bool pdl_enabled() { return true; }
#endif

int* device_status_word() {
    int* w = g_status_word.load(std::memory_order_acquire);
    if (w != nullptr) return w;
    std::lock_guard<std::mutex> lock(g_status_mutex);
    w = g_status_word.load(std::memory_order_relaxed);
    if (w != nullptr) return w;
    // A caller may be capturing a CUDA graph; the one allocation of pinned
    // host memory is made in relaxed capture mode, which allows it.
    cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
    cudaThreadExchangeStreamCaptureMode(&mode);
    void* p = nullptr;
    const cudaError_t e = cudaHostAlloc(&p, sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable);
    cudaThreadExchangeStreamCaptureMode(&mode);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error(AKO_B200_ERR_CUDA, "status word: cudaHostAlloc failed: %s", cudaGetErrorString(e));
        return nullptr;
    }
    w = static_cast<int*>(p);
    *reinterpret_cast<volatile int*>(w) = 0;
    g_status_word.store(w, std::memory_order_release);
    return w;
}

int refuse_if_wait_expired(const char* op) {
    const int* w = g_status_word.load(std::memory_order_acquire);
    if (w == nullptr || *reinterpret_cast<const volatile int*>(w) == 0) return AKO_B200_OK;
    return set_error(AKO_B200_ERR_WAIT_EXPIRED,
                     "%s: refused: a bounded wait for a bulk copy ran out in an earlier RMSNorm launch (its "
                     "unwritten rows hold NaN); ako_b200_take_device_status reports and clears it",
                     op);
}

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
        case AKO_B200_ERR_WAIT_EXPIRED: return "AKO_B200_ERR_WAIT_EXPIRED";
        default: return "AKO_B200_ERR_UNKNOWN";
    }
}

const char* ako_b200_last_error(void) { return ako_b200::g_last_error; }

int ako_b200_take_device_status(int* status) {
    using namespace ako_b200;
    clear_error();
    if (status == nullptr) return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "status is a null pointer");
    int* w = g_status_word.load(std::memory_order_acquire);
    if (w == nullptr) {  // no persistent kernel has run in this process
        *status = 0;
        return AKO_B200_OK;
    }
    const cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return set_error(AKO_B200_ERR_CUDA, "device status: %s", cudaGetErrorString(e));
    volatile int* v = w;
    *status = *v;
    *v = 0;
    return AKO_B200_OK;
}

#ifdef AKO_B200_MEASUREMENT
int ako_b200_set_pdl(int enable) { return ako_b200::g_pdl.exchange(enable ? 1 : 0); }
#endif

}  // extern "C"
