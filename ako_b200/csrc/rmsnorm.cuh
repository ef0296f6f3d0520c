// RMSNorm and fused residual-add RMSNorm kernels for sm_100a.
//
// Definition (reference ako/ops/rmsnorm_ref.py:8-23 and :26-50):
//   r'  = round_T(x + residual)                       (residual variant only)
//   var = sum(v * v) / H          over the row, fp32, v = float(x) or float(r')
//   inv = 1 / sqrt(var + eps)     (two IEEE roundings, as torch.rsqrt on CPU)
//   y   = round_T((v * inv) * w)  (two fp32 roundings, in the reference order)
// Squares are rounded before they are summed (the reference materializes
// x.pow(2)); only the summation order differs from the reference.
//
// Two kernels:
//  * rms_rows_kernel: row-resident. TPR threads own a row; each thread holds
//    NV 16-byte vectors of it in registers (packed in the storage dtype), so
//    the row is read from HBM once and written once. TPR == 32 puts one row
//    on each warp (4 rows per 128-thread CTA, shuffle-only reduction); larger
//    TPR puts one row on a CTA (shuffle + one shared-memory exchange).
//  * rms_generic_kernel: any width and alignment. One CTA per row, scalar
//    accesses, two passes; the second pass re-reads the row (an L2 hit for
//    rows up to the L2 size).
#pragma once

#include "common.cuh"
#include "host.hpp"

namespace ako_b200 {

struct RmsArgs {
    const void* x;
    int64_t sx;
    const void* r;
    int64_t sr;
    const void* w;
    int wdtype;
    void* y;
    int64_t sy;
    void* ro;
    int64_t sro;
    int64_t rows;
    int h;
    float eps;
};

template <int TPR>
struct RmsShape {
    static constexpr int kThreads = TPR <= 32 ? 128 : TPR;
    static constexpr int kRowsPerCta = kThreads / TPR;
};

template <typename T, int TPR, int NV, bool RES>
__global__ void __launch_bounds__(RmsShape<TPR>::kThreads)
rms_rows_kernel(const RmsArgs a) {
    constexpr int VEC = 16 / sizeof(T);
    constexpr int THREADS = RmsShape<TPR>::kThreads;
    constexpr int ROWS = RmsShape<TPR>::kRowsPerCta;
    using P = Packed<T, VEC>;
    __shared__ float scratch[THREADS / 32 > 0 ? THREADS / 32 : 1];

    const int lane = threadIdx.x % TPR;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * ROWS + threadIdx.x / TPR;
    // Warp-per-row CTAs reduce with shuffles only, so a warp whose row is past
    // the end can leave; CTA-per-row grids have exactly one CTA per row.
    if (ROWS > 1 && row >= a.rows) return;

    const T* xr = static_cast<const T*>(a.x) + row * a.sx;
    P v[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        const int col = (j * TPR + lane) * VEC;
        if (col < a.h) v[j] = ld_stream<T, VEC>(xr + col);
    }

    if constexpr (RES) {
        const T* rr = static_cast<const T*>(a.r) + row * a.sr;
        T* ro = static_cast<T*>(a.ro) + row * a.sro;
        P rv[NV];
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int col = (j * TPR + lane) * VEC;
            if (col < a.h) rv[j] = ld_stream<T, VEC>(rr + col);
        }
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int col = (j * TPR + lane) * VEC;
            if (col < a.h) {
#pragma unroll
                for (int e = 0; e < VEC; ++e)
                    v[j].v[e] = from_f32<T>(__fadd_rn(to_f32(v[j].v[e]), to_f32(rv[j].v[e])));
                st_global<T, VEC>(ro + col, v[j]);
            }
        }
    }

    // Squares are rounded, then summed pairwise: within a vector, across the
    // thread's vectors, across lanes, across warps.
    float part[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        const int col = (j * TPR + lane) * VEC;
        float sq[VEC];
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
            const float f = to_f32(v[j].v[e]);
            sq[e] = __fmul_rn(f, f);
        }
        part[j] = col < a.h ? tree_sum<VEC>(sq) : 0.0f;
    }
    const float acc = tree_sum<NV>(part);
    float total;
    if constexpr (TPR <= 32) {
        total = warp_sum<TPR>(acc);
    } else {
        total = block_sum<THREADS>(acc, scratch);
    }
    const float mean = __fdiv_rn(total, static_cast<float>(a.h));
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));

    T* yr = static_cast<T*>(a.y) + row * a.sy;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        const int col = (j * TPR + lane) * VEC;
        if (col < a.h) {
            float w[VEC];
            load_weight_vec<VEC>(a.w, a.wdtype, col, w);
            P o;
#pragma unroll
            for (int e = 0; e < VEC; ++e)
                o.v[e] = from_f32<T>(__fmul_rn(__fmul_rn(to_f32(v[j].v[e]), inv), w[e]));
            st_global<T, VEC>(yr + col, o);
        }
    }
}

constexpr int kGenericThreads = 256;

template <typename T, bool RES>
__global__ void __launch_bounds__(kGenericThreads) rms_generic_kernel(const RmsArgs a) {
    __shared__ float scratch[kGenericThreads / 32];
    const int64_t row = blockIdx.x;
    const T* xr = static_cast<const T*>(a.x) + row * a.sx;
    const T* rr = RES ? static_cast<const T*>(a.r) + row * a.sr : nullptr;
    T* ro = RES ? static_cast<T*>(a.ro) + row * a.sro : nullptr;

    // Rounded squares accumulated in fp64 per thread (any row length stays
    // within one fp32 rounding of the exact sum), then pairwise across threads.
    double acc = 0.0;
    for (int col = threadIdx.x; col < a.h; col += kGenericThreads) {
        float f = to_f32(xr[col]);
        if constexpr (RES) {
            const T s = from_f32<T>(__fadd_rn(f, to_f32(rr[col])));
            ro[col] = s;
            f = to_f32(s);
        }
        acc += static_cast<double>(__fmul_rn(f, f));
    }
    const float total = block_sum<kGenericThreads>(static_cast<float>(acc), scratch);
    const float mean = __fdiv_rn(total, static_cast<float>(a.h));
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));

    T* yr = static_cast<T*>(a.y) + row * a.sy;
    for (int col = threadIdx.x; col < a.h; col += kGenericThreads) {
        // The residual pass reads back what this same thread stored above.
        const float f = RES ? to_f32(ro[col]) : to_f32(xr[col]);
        yr[col] = from_f32<T>(__fmul_rn(__fmul_rn(f, inv), load_weight(a.w, a.wdtype, col)));
    }
}

#define AKO_RMS_CASE(T, RES, TPR, NV)                                                               \
    case TPR * 16 + NV: {                                                                           \
        constexpr int rows_per_cta = RmsShape<TPR>::kRowsPerCta;                                    \
        const int64_t grid = (a.rows + rows_per_cta - 1) / rows_per_cta;                            \
        rms_rows_kernel<T, TPR, NV, RES><<<static_cast<unsigned>(grid), RmsShape<TPR>::kThreads, 0, \
                                           st>>>(a);                                                \
        return check_launch(RES ? "rmsnorm_residual" : "rmsnorm");                                  \
    }

#define AKO_RMS_ALL_CASES(T, RES)                                                                    \
    AKO_RMS_CASE(T, RES, 32, 1)                                                                      \
    AKO_RMS_CASE(T, RES, 32, 2)                                                                      \
    AKO_RMS_CASE(T, RES, 32, 4)                                                                      \
    AKO_RMS_CASE(T, RES, 32, 8)                                                                      \
    AKO_RMS_CASE(T, RES, 64, 2)                                                                      \
    AKO_RMS_CASE(T, RES, 64, 4)                                                                      \
    AKO_RMS_CASE(T, RES, 64, 8)                                                                      \
    AKO_RMS_CASE(T, RES, 128, 1)                                                                     \
    AKO_RMS_CASE(T, RES, 128, 2)                                                                     \
    AKO_RMS_CASE(T, RES, 128, 4)                                                                     \
    AKO_RMS_CASE(T, RES, 128, 8)                                                                     \
    AKO_RMS_CASE(T, RES, 256, 1)                                                                     \
    AKO_RMS_CASE(T, RES, 256, 2)                                                                     \
    AKO_RMS_CASE(T, RES, 256, 4)                                                                     \
    AKO_RMS_CASE(T, RES, 256, 8)                                                                     \
    AKO_RMS_CASE(T, RES, 512, 1)                                                                     \
    AKO_RMS_CASE(T, RES, 512, 2)                                                                     \
    AKO_RMS_CASE(T, RES, 512, 4)                                                                     \
    AKO_RMS_CASE(T, RES, 512, 8)                                                                     \
    AKO_RMS_CASE(T, RES, 1024, 2)                                                                    \
    AKO_RMS_CASE(T, RES, 1024, 4)                                                                    \
    AKO_RMS_CASE(T, RES, 1024, 8)

// Launches the row-resident kernel for (tpr, nv); returns -1 when that pair
// is not instantiated.
template <typename T, bool RES>
int launch_rms_rows(const RmsArgs& a, int tpr, int nv, cudaStream_t st) {
    switch (tpr * 16 + nv) {
        AKO_RMS_ALL_CASES(T, RES)
        default: return -1;
    }
}

template <typename T, bool RES>
int launch_rms_generic(const RmsArgs& a, cudaStream_t st) {
    rms_generic_kernel<T, RES><<<static_cast<unsigned>(a.rows), kGenericThreads, 0, st>>>(a);
    return check_launch(RES ? "rmsnorm_residual(generic)" : "rmsnorm(generic)");
}

// Instantiated once per dtype in rmsnorm_{f32,f16,bf16}.cu (compiled in parallel).
#define AKO_RMS_DECLARE(T, KW)                                                        \
    KW template int launch_rms_rows<T, false>(const RmsArgs&, int, int, cudaStream_t); \
    KW template int launch_rms_rows<T, true>(const RmsArgs&, int, int, cudaStream_t);  \
    KW template int launch_rms_generic<T, false>(const RmsArgs&, cudaStream_t);        \
    KW template int launch_rms_generic<T, true>(const RmsArgs&, cudaStream_t);

#ifndef AKO_RMS_INSTANTIATING
AKO_RMS_DECLARE(float, extern)
AKO_RMS_DECLARE(__half, extern)
AKO_RMS_DECLARE(__nv_bfloat16, extern)
#endif

}  // namespace ako_b200
