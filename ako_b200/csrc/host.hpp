// Host-side helpers shared by the C-ABI entry points: per-thread error text,
// launch checking and alignment tests.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "ako_b200.h"

namespace ako_b200 {

// Records a printf-style message for ako_b200_last_error() and returns `status`.
int set_error(int status, const char* fmt, ...);

// Clears the calling thread's message; returns AKO_B200_OK.
int clear_error();

// Converts the result of the launch just issued into a status code.
int check_launch(const char* kernel);

// Streaming-multiprocessor count of the current device (cached per device).
int sm_count();

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
