// Host-side helpers shared by the C-ABI entry points: per-thread error text,
// launch checking, alignment tests, the persistent kernels' status word, and
// the launch overrides of measurement builds.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "ako_b200.h"

// Launch overrides (forced shapes, kernels, programmatic launch, wait limits)
// exist only in the measurement build of the library (libako_b200_measure.so,
// compiled with AKO_B200_MEASUREMENT, setters in ako_b200_measure.h). The
// product library compiles each override as a constant at its built-in
// value, so no call can change which kernel another caller's call runs.
#ifdef AKO_B200_MEASUREMENT
#include "ako_b200_measure.h"
#define AKO_B200_OVERRIDE
#else
#define AKO_B200_OVERRIDE constexpr
#endif

namespace ako_b200 {

// Records a printf-style message for ako_b200_last_error() and returns `status`.
int set_error(int status, const char* fmt, ...);

// Clears the calling thread's message; returns AKO_B200_OK.
int clear_error();

// Converts the result of the launch just issued into a status code.
int check_launch(const char* kernel);

// Streaming-multiprocessor count of the current device (cached per device).
int sm_count();

// Whether launches carry programmatic stream serialization (see launch_ex).
bool pdl_enabled();

// Host-mapped status word of the persistent RMSNorm kernels, allocated
// (pinned, mapped, portable to every device) on first use; nullptr if that
// allocation failed, with the error recorded. A kernel whose bounded wait
// for a bulk copy runs out stores kStatusWaitTimeout there with a plain
// system-scope store; the host reads it without synchronizing.
int* device_status_word();

// AKO_B200_ERR_WAIT_EXPIRED (with a message naming `op`) while the status
// word holds an unreported expiry, else AKO_B200_OK. Every entry point that
// launches checks it first, so an expiry is never followed silently by more
// work; ako_b200_take_device_status clears it.
int refuse_if_wait_expired(const char* op);

// Launches kernel(a) on `grid` x `block` with `smem` bytes of dynamic shared
// memory, in clusters of `cluster` CTAs along x when cluster > 1. With
// programmatic dependent launch enabled, the kernel may begin while the
// previous kernel in the stream drains; every kernel of this library waits
// for that grid (griddepcontrol.wait) before its first global memory access,
// so results are unchanged and only the launch gap is hidden.
template <typename Args>
int launch_ex(void (*kernel)(Args), dim3 grid, dim3 block, size_t smem, int cluster, cudaStream_t st, const Args& a,
              const char* name) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int n = 0;
    if (cluster > 1) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = cluster;
        attr[n].val.clusterDim.y = 1;
        attr[n].val.clusterDim.z = 1;
        ++n;
    }
    if (pdl_enabled()) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    cfg.attrs = n ? attr : nullptr;
    cfg.numAttrs = n;
    const cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, a);
    if (err != cudaSuccess) {
        cudaGetLastError();
        return set_error(AKO_B200_ERR_CUDA, "%s: launch failed: %s", name, cudaGetErrorString(err));
    }
    return check_launch(name);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// True when a row stride of `stride` elements of `elem` bytes keeps every row
// start on a 16-byte boundary (strides of single-row operands never matter).
inline bool stride_ok16(int64_t stride, int64_t rows, int elem) {
    return rows <= 1 || ((stride * elem) & 15) == 0;
}

inline int dtype_size(int dtype) {
    switch (dtype) {
        case AKO_B200_F32: return 4;
        case AKO_B200_F16: return 2;
        case AKO_B200_BF16: return 2;
        default: return 0;
    }
}

}  // namespace ako_b200
