// SwiGLU activation for sm_100a, plus its C-ABI entry point.
//
// Definition (reference ako/ops/swiglu_ref.py:16-32, F.silu on fp32):
//   y = round_T( (g / (1 + exp(-g))) * u ),  g = float(gate), u = float(up)
// with IEEE division and one fp32 rounding per operation, as torch's CPU silu
// kernel evaluates it. expf is CUDA's (not the fast-math intrinsic).
//
// Element-wise over an (n_rows x hidden_dim) matrix whose three operands have
// independent row strides (the packed [M, 2F] layout is two strided views).
// Work is a flat sequence of 16-byte vectors; a grid of a few CTAs per SM
// strides over it, each thread keeping UNROLL vectors of both inputs in
// flight before it computes.
#include <climits>

#include "common.cuh"
#include "host.hpp"

namespace ako_b200 {
namespace {

struct SwigluArgs {
    const void* g;
    int64_t sg;
    const void* u;
    int64_t su;
    void* y;
    int64_t sy;
    int64_t total;  // vectors (or elements, scalar path) in the matrix
    int64_t per_row;
};

constexpr int kThreads = 256;

__device__ __forceinline__ float silu_mul(float g, float u) {
    const float s = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
    return __fmul_rn(s, u);
}

// FLAT: all three operands are dense (row stride == hidden_dim), so vector
// i sits at element i * VEC of each. Otherwise rows are recovered with a
// 32-bit (NARROW) or 64-bit division.
template <typename T, int VEC, int UNROLL, bool FLAT, bool NARROW>
__global__ void __launch_bounds__(kThreads) swiglu_kernel(const SwigluArgs a) {
    using P = Packed<T, VEC>;
    const T* gp = static_cast<const T*>(a.g);
    const T* up = static_cast<const T*>(a.u);
    T* yp = static_cast<T*>(a.y);
    const int64_t step = static_cast<int64_t>(gridDim.x) * kThreads * UNROLL;
    for (int64_t base = static_cast<int64_t>(blockIdx.x) * kThreads * UNROLL + threadIdx.x; base < a.total;
         base += step) {
        P g[UNROLL], u[UNROLL];
        int64_t yo[UNROLL];
#pragma unroll
        for (int k = 0; k < UNROLL; ++k) {
            const int64_t i = base + static_cast<int64_t>(k) * kThreads;
            if (i < a.total) {
                int64_t go, uo;
                if constexpr (FLAT) {
                    go = uo = yo[k] = i * VEC;
                } else {
                    int64_t row, col;
                    if constexpr (NARROW) {
                        const uint32_t r32 = static_cast<uint32_t>(i) / static_cast<uint32_t>(a.per_row);
                        row = r32;
                        col = static_cast<int64_t>(static_cast<uint32_t>(i) - r32 * static_cast<uint32_t>(a.per_row));
                    } else {
                        row = i / a.per_row;
                        col = i - row * a.per_row;
                    }
                    col *= VEC;
                    go = row * a.sg + col;
                    uo = row * a.su + col;
                    yo[k] = row * a.sy + col;
                }
                if constexpr (VEC * sizeof(T) == 16) {
                    g[k] = ld_stream<T, VEC>(gp + go);
                    u[k] = ld_stream<T, VEC>(up + uo);
                } else {
                    g[k] = ld_cached<T, VEC>(gp + go);
                    u[k] = ld_cached<T, VEC>(up + uo);
                }
            }
        }
#pragma unroll
        for (int k = 0; k < UNROLL; ++k) {
            const int64_t i = base + static_cast<int64_t>(k) * kThreads;
            if (i < a.total) {
                P o;
#pragma unroll
                for (int e = 0; e < VEC; ++e) o.v[e] = from_f32<T>(silu_mul(to_f32(g[k].v[e]), to_f32(u[k].v[e])));
                st_global<T, VEC>(yp + yo[k], o);
            }
        }
    }
}

template <typename T, int VEC, int UNROLL>
int launch(const SwigluArgs& a, bool flat, cudaStream_t st) {
    const int64_t per_cta = static_cast<int64_t>(kThreads) * UNROLL;
    int64_t grid = (a.total + per_cta - 1) / per_cta;
    const int64_t cap = static_cast<int64_t>(sm_count()) * 8;  // 8 CTAs of 256 threads fill an SM
    if (grid > cap) grid = cap;
    const unsigned g = static_cast<unsigned>(grid);
    if (flat) {
        swiglu_kernel<T, VEC, UNROLL, true, true><<<g, kThreads, 0, st>>>(a);
    } else if (a.total <= static_cast<int64_t>(UINT_MAX)) {
        swiglu_kernel<T, VEC, UNROLL, false, true><<<g, kThreads, 0, st>>>(a);
    } else {
        swiglu_kernel<T, VEC, UNROLL, false, false><<<g, kThreads, 0, st>>>(a);
    }
    return check_launch("swiglu");
}

template <typename T>
int run(SwigluArgs a, int64_t rows, int64_t h, bool vector_ok, bool flat, cudaStream_t st) {
    constexpr int VEC = 16 / sizeof(T);
    if (vector_ok) {
        a.per_row = h / VEC;
        a.total = rows * a.per_row;
        // Small problems (decode rows) spread over more CTAs; large ones keep
        // four vectors per thread in flight.
        if (a.total < static_cast<int64_t>(sm_count()) * kThreads * 4) return launch<T, VEC, 1>(a, flat, st);
        return launch<T, VEC, 4>(a, flat, st);
    }
    a.per_row = h;
    a.total = rows * h;
    return launch<T, 1, 4>(a, flat, st);
}

}  // namespace
}  // namespace ako_b200

using namespace ako_b200;

extern "C" int ako_b200_swiglu(const void* gate, int64_t gate_row_stride, const void* up, int64_t up_row_stride,
                               void* y, int64_t y_row_stride, int64_t n_rows, int64_t hidden_dim, int dtype,
                               void* stream) {
    clear_error();
    const char* op = "ako_b200_swiglu";
    const int es = dtype_size(dtype);
    if (es == 0) return set_error(AKO_B200_ERR_UNSUPPORTED_DTYPE, "%s: unsupported dtype code %d", op, dtype);
    if (n_rows < 0 || hidden_dim < 0)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: negative size", op);
    if (n_rows == 0 || hidden_dim == 0) return AKO_B200_OK;
    if (gate == nullptr || up == nullptr || y == nullptr)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: null pointer", op);
    if (n_rows > 1 && (gate_row_stride < hidden_dim || up_row_stride < hidden_dim || y_row_stride < hidden_dim))
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: a row stride is smaller than hidden_dim %lld", op,
                         static_cast<long long>(hidden_dim));
    if (n_rows == 1) gate_row_stride = up_row_stride = y_row_stride = hidden_dim;

    const bool flat = gate_row_stride == hidden_dim && up_row_stride == hidden_dim && y_row_stride == hidden_dim;
    const bool vector_ok = (hidden_dim * es) % 16 == 0 && aligned16(gate) && aligned16(up) && aligned16(y) &&
                           stride_ok16(gate_row_stride, n_rows, es) && stride_ok16(up_row_stride, n_rows, es) &&
                           stride_ok16(y_row_stride, n_rows, es);
    SwigluArgs a{gate, gate_row_stride, up, up_row_stride, y, y_row_stride, 0, 0};
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (dtype) {
        case AKO_B200_F32: return run<float>(a, n_rows, hidden_dim, vector_ok, flat, st);
        case AKO_B200_F16: return run<__half>(a, n_rows, hidden_dim, vector_ok, flat, st);
        default: return run<__nv_bfloat16>(a, n_rows, hidden_dim, vector_ok, flat, st);
    }
}
