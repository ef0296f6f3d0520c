// RMSNorm and fused residual-add RMSNorm kernels for sm_100a.
//
// Definition (reference ako/ops/rmsnorm_ref.py:8-23 and :26-50):
//   r'  = round_T(x + residual)                       (residual variant only)
//   var = sum(v * v) / H          over the row, fp32, v = float(x) or float(r')
//   inv = 1 / sqrt(var + eps)     (two IEEE roundings, as torch.rsqrt on CPU)
//   y   = round_T((v * inv) * w)  (two fp32 roundings, in the reference order)
// Squares are rounded before they are summed (the reference materializes
// x.pow(2)); only the summation order differs from the reference. The
// vector kernels share one summation order that depends only on the row
// width (common.cuh, "fixed-order sums"), so a row's output bits do not
// depend on the launch shape or on how many rows the call has: a token
// normalized in a prefill batch and alone in a decode step gives the same
// bits.
//
// Two kernels:
//  * rms_rows_kernel: row-resident. TPR threads own a row; each thread holds
//    NV 16-byte vectors of it in registers (packed in the storage dtype), so
//    the row is read from HBM once and written once. TPR == 32 puts one row
//    on each warp (4 rows per 128-thread CTA, shuffle-only reduction); larger
//    TPR puts one row on a CTA (shuffle + one shared-memory exchange).
//  * rms_generic_kernel: any width and alignment. One CTA per row, two
//    passes (the second re-reads the row, an L2 hit for rows up to the L2
//    size); when all of a row's pointers share one offset within 16 bytes,
//    16-byte accesses for its aligned middle and element accesses for the
//    ends, else element accesses throughout.
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
    float inv_h;  // 1 / h when h is a power of two (then exact), else 0
};

// 1 / sqrt(sum / h + eps) with the reference's roundings: the mean is one
// IEEE quotient (a product with inv_h when h is a power of two: scaling by a
// power of two rounds the same real number), then an IEEE square root and
// the correctly rounded reciprocal, which is the IEEE quotient 1 / s.
__device__ __forceinline__ float rms_inv(float total, const RmsArgs& a) {
    const float mean = a.inv_h != 0.0f ? __fmul_rn(total, a.inv_h) : __fdiv_rn(total, static_cast<float>(a.h));
    return __frcp_rn(__fsqrt_rn(__fadd_rn(mean, a.eps)));
}

template <int TPR>
struct RmsShape {
    static_assert(TPR % 32 == 0, "a row's threads must be whole warps (fixed summation order)");
    static constexpr int kThreads = TPR <= 32 ? 128 : TPR;
    static constexpr int kRowsPerCta = kThreads / TPR;
};

constexpr int pow2_ceil(int n) { return n <= 1 ? 1 : 2 * pow2_ceil((n + 1) / 2); }

// The weight is held in registers (4 per vector) by shapes with at most
// WEIGHT_NV vectors per thread, or at most WEIGHT_CTA_VECTORS vectors per
// CTA (few threads, many vectors each: the register file is not what bounds
// their occupancy).
constexpr int WEIGHT_NV = 2;
constexpr int WEIGHT_CTA_VECTORS = 1024;

// CTAs per SM the register allocation must leave room for (the second
// launch bound; 0 leaves it out). 512-thread CTAs with the weight in
// registers take 46-48 registers a thread unbounded, which fits two per SM;
// at 40 three fit, and rows of 1024 bf16 vectors run 5-7% faster (measured
// on B200). Other shapes are faster unbounded: an explicit bound of 1
// changes their code even where it does not bind.
template <int TPR, int NV>
constexpr int rms_min_ctas() {
    return (RmsShape<TPR>::kThreads == 512 && NV <= WEIGHT_NV) ? 3 : 0;
}

// CLUSTER > 1: a row is split into CLUSTER equal slices, one per CTA of a
// thread-block cluster; CTA partial sums are exchanged through distributed
// shared memory, so each CTA holds only H / CLUSTER elements in registers.
template <typename T, int TPR, int NV, bool RES, int CLUSTER>
__global__ void __launch_bounds__(RmsShape<TPR>::kThreads, rms_min_ctas<TPR, NV>())
rms_rows_kernel(const RmsArgs a) {
    constexpr int VEC = 16 / sizeof(T);
    constexpr int THREADS = RmsShape<TPR>::kThreads;
    constexpr int ROWS = RmsShape<TPR>::kRowsPerCta;
    static_assert(CLUSTER == 1 || ROWS == 1, "clusters split CTA-per-row shapes only");
    constexpr int WARPS = THREADS / 32;
    // Group sums of the CTA's row slice (CTA-per-row shapes): NV per warp.
    constexpr int GROUPS = TPR > 32 ? NV * WARPS : 1;
    using P = Packed<T, VEC>;
    __shared__ float gsum[GROUPS];
    pdl_enter();

    const int lane = threadIdx.x % TPR;
    const int64_t row = CLUSTER > 1 ? static_cast<int64_t>(blockIdx.x / CLUSTER)
                                    : static_cast<int64_t>(blockIdx.x) * ROWS + threadIdx.x / TPR;
    // Warp-per-row CTAs reduce with shuffles only, so a warp whose row is past
    // the end can leave; CTA-per-row grids have exactly one CTA per row slice.
    if (ROWS > 1 && row >= a.rows) return;
    // This CTA's slice of the row: columns [c0, c0 + width).
    const int width = CLUSTER > 1 ? a.h / CLUSTER : a.h;
    const int c0 = CLUSTER > 1 ? static_cast<int>(cluster_ctarank()) * width : 0;

    const T* xr = static_cast<const T*>(a.x) + row * a.sx + c0;
    P v[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        const int col = (j * TPR + lane) * VEC;
        if (col < width) v[j] = ld_stream<T, VEC>(xr + col);
    }
    // The weight is needed only after the reduction. Fetching it there puts a
    // second memory round trip on every row's critical path (measured: up to
    // 20% of the kernel on 8192 x 2048 bf16 rows). When it has the row's dtype
    // (the usual case) it is loaded now, next to the row, and held packed like
    // the row (4 registers per vector); other weight dtypes, and shapes whose
    // registers are better spent on occupancy, prefetch it to L1 instead.
    // Plain fp32 rows on the fitted 320- and 384-thread shapes also hold it:
    // prefetched, those compiled to 32 registers and moved 2.2x the row's
    // bytes through L2, and 32768 x 4608 timed 0.73 of peak against 1.05
    // holding it (5120 wide 0.88 -> 1.05; 448 threads were slower holding it).
    constexpr bool kWeightRegs = NV <= WEIGHT_NV || THREADS * NV <= WEIGHT_CTA_VECTORS ||
                                 (sizeof(T) == 4 && !RES && (TPR & (TPR - 1)) != 0 && THREADS * NV <= 1536);
    // Shapes that cannot spare the registers copy it into shared memory now
    // instead (cp.async: no registers held, each thread reads back only its
    // own vectors), up to 32 KB a CTA; 512 x 4 bf16 rows of 16384 took
    // 14.7 us at 512 rows prefetching it to L1 and loading it after the
    // reduction, against 13.2 us for AKO's Triton kernel, which loads it
    // with the row.
    constexpr bool kWeightSmem = !kWeightRegs && THREADS * NV * 16 <= 32 * 1024;
    P wv[kWeightRegs ? NV : 1];
    __shared__ __align__(16) P wsm[kWeightSmem ? NV * THREADS : 1];
    bool w_regs = false;
    if constexpr (kWeightRegs) {
        w_regs = a.wdtype == dtype_code<T>();
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int col = (j * TPR + lane) * VEC;
            if (col < width) {
                if (w_regs) {
                    wv[j] = ld_cached<T, VEC>(static_cast<const T*>(a.w) + c0 + col);
                } else {
                    prefetch_weight(a.w, a.wdtype, c0 + col);
                }
            }
        }
    } else if constexpr (kWeightSmem) {
        w_regs = a.wdtype == dtype_code<T>();
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int col = (j * TPR + lane) * VEC;
            if (col < width) {
                if (w_regs) {
                    cp_async16(&wsm[j * THREADS + threadIdx.x], static_cast<const T*>(a.w) + c0 + col);
                } else {
                    prefetch_weight(a.w, a.wdtype, c0 + col);
                }
            }
        }
        cp_async_commit();
    } else {
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int col = (j * TPR + lane) * VEC;
            if (col < width) prefetch_weight(a.w, a.wdtype, c0 + col);
        }
    }

    if constexpr (RES) {
        const T* rr = static_cast<const T*>(a.r) + row * a.sr + c0;
        T* ro = static_cast<T*>(a.ro) + row * a.sro + c0;
        P rv[NV];
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int col = (j * TPR + lane) * VEC;
            if (col < width) rv[j] = ld_stream<T, VEC>(rr + col);
        }
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int col = (j * TPR + lane) * VEC;
            if (col < width) {
#pragma unroll
                for (int e = 0; e < VEC; e += 2) {
                    const float2 xa = get2<T, VEC>(v[j], e);
                    const float2 ra = get2<T, VEC>(rv[j], e);
                    put2<T, VEC>(v[j], e, __fadd_rn(xa.x, ra.x), __fadd_rn(xa.y, ra.y));
                }
                st_global<T, VEC>(ro + col, v[j]);
            }
        }
    }

    // Squares are rounded, then summed in the fixed order: within a vector,
    // across each 32-vector group's lanes, across the groups.
    float part[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        const int col = (j * TPR + lane) * VEC;
        float sq[VEC];
#pragma unroll
        for (int e = 0; e < VEC; e += 2) {
            const float2 f = get2<T, VEC>(v[j], e);
            sq[e] = __fmul_rn(f.x, f.x);
            sq[e + 1] = __fmul_rn(f.y, f.y);
        }
        part[j] = col < width ? tree_sum<VEC>(sq) : 0.0f;
    }
    float total;
    if constexpr (TPR <= 32) {
        total = warp_row_sum<NV>(part);
    } else {
        // Every warp folds the row's group sums itself, so no second barrier
        // or broadcast is needed.
        constexpr int K = pow2_ceil((CLUSTER * GROUPS + 31) / 32);
        store_group_sums<NV>(fold_groups_scatter<NV>(part), gsum, WARPS);
        if constexpr (CLUSTER == 1) {
            __syncthreads();
            total = fold_group_sums<K>(GROUPS, [&](int i) { return gsum[i]; });
        } else {
            // Group i of the row is group i % sg of the slice of CTA i / sg
            // (the host splits rows into slices of whole 32-vector groups).
            // The second cluster barrier is split: arrive now, wait before
            // exit, so no CTA leaves while another may still read its shared
            // memory.
            const int sg = width / VEC / 32;
            cluster_sync_all();
            total = fold_group_sums<K>(CLUSTER * sg, [&](int i) {
                return ld_dsmem_f32(&gsum[i % sg], static_cast<unsigned>(i / sg));
            });
            cluster_arrive();
        }
    }
    const float inv = rms_inv(total, a);
    if constexpr (kWeightSmem) cp_async_wait_all();

    T* yr = static_cast<T*>(a.y) + row * a.sy + c0;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        const int col = (j * TPR + lane) * VEC;
        if (col < width) {
            P o;
            if (kWeightRegs && w_regs) {
#pragma unroll
                for (int e = 0; e < VEC; e += 2) {
                    const float2 f = get2<T, VEC>(v[j], e);
                    const float2 w = get2<T, VEC>(wv[kWeightRegs ? j : 0], e);
                    put2<T, VEC>(o, e, __fmul_rn(__fmul_rn(f.x, inv), w.x), __fmul_rn(__fmul_rn(f.y, inv), w.y));
                }
            } else if (kWeightSmem && w_regs) {
                const P wj = wsm[kWeightSmem ? j * THREADS + threadIdx.x : 0];
#pragma unroll
                for (int e = 0; e < VEC; e += 2) {
                    const float2 f = get2<T, VEC>(v[j], e);
                    const float2 w = get2<T, VEC>(wj, e);
                    put2<T, VEC>(o, e, __fmul_rn(__fmul_rn(f.x, inv), w.x), __fmul_rn(__fmul_rn(f.y, inv), w.y));
                }
            } else {
                float w[VEC];
                load_weight_vec<VEC>(a.w, a.wdtype, c0 + col, w);
#pragma unroll
                for (int e = 0; e < VEC; e += 2) {
                    const float2 f = get2<T, VEC>(v[j], e);
                    put2<T, VEC>(o, e, __fmul_rn(__fmul_rn(f.x, inv), w[e]), __fmul_rn(__fmul_rn(f.y, inv), w[e + 1]));
                }
            }
            st_global<T, VEC>(yr + col, o);
        }
    }
    if constexpr (CLUSTER > 1) cluster_wait();
}

constexpr int kGenericThreads = 256;

// 16 bytes starting MIS bytes into the aligned 16-byte block p[0] (MIS even,
// p[1] the next block): each output word joins two neighbouring words.
template <int MIS>
__device__ __forceinline__ uint4 shifted16(const uint4* p) {
    if constexpr (MIS == 0) {
        return *p;
    } else {
        const uint4 lo = p[0], hi = p[1];
        const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
        constexpr int Q = MIS / 4, SH = (MIS % 4) * 8;
        uint32_t o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i] = SH == 0 ? w[i + Q] : __funnelshift_r(w[i + Q], w[i + Q + 1], SH);
        return make_uint4(o[0], o[1], o[2], o[3]);
    }
}

// Vector body of the generic kernel's output pass, for a weight of the row's
// dtype at byte misalignment MIS (see rms_generic_kernel). A vector whose
// aligned blocks reach outside the weight tensor (only the first or last
// can, when the weight itself is not 16-byte aligned at its ends) reads its
// weights element by element, so every access stays inside the tensor.
template <typename T, bool RES, int MIS, int TPR>
__device__ __forceinline__ void generic_body_shifted(const RmsArgs& a, const T* xr, const T* ro, T* yr, int head,
                                                     int nvec, float inv, const uint4* wv, int lane) {
    constexpr int VEC = 16 / sizeof(T);
    using P = Packed<T, VEC>;
    const uintptr_t w_begin = reinterpret_cast<uintptr_t>(a.w);
    const uintptr_t w_end = w_begin + static_cast<uintptr_t>(a.h) * sizeof(T);
    for (int v = lane; v < nvec; v += TPR) {
        const int col = head + v * VEC;
        const P xv = RES ? ld_cached<T, VEC>(ro + col) : ld_cached<T, VEC>(xr + col);
        const uintptr_t blk = reinterpret_cast<uintptr_t>(wv + v);
        P o;
        if (blk >= w_begin && blk + (MIS == 0 ? 16 : 32) <= w_end) {
            const uint4 wr = shifted16<MIS>(wv + v);
            const P wp = *reinterpret_cast<const P*>(&wr);
#pragma unroll
            for (int e = 0; e < VEC; e += 2) {
                const float2 f = get2<T, VEC>(xv, e);
                const float2 w = get2<T, VEC>(wp, e);
                put2<T, VEC>(o, e, __fmul_rn(__fmul_rn(f.x, inv), w.x), __fmul_rn(__fmul_rn(f.y, inv), w.y));
            }
        } else {
#pragma unroll
            for (int e = 0; e < VEC; e += 2) {
                const float2 f = get2<T, VEC>(xv, e);
                put2<T, VEC>(o, e, __fmul_rn(__fmul_rn(f.x, inv), load_weight(a.w, a.wdtype, col + e)),
                             __fmul_rn(__fmul_rn(f.y, inv), load_weight(a.w, a.wdtype, col + e + 1)));
            }
        }
        st_global<T, VEC>(yr + col, o);
    }
}

// TPR threads per row: 256 (one CTA per row), or 32 for narrow rows (a warp
// per row, four rows per 128-thread CTA, shuffle-only reduction).
template <int TPR>
constexpr int generic_threads() {
    return TPR == 32 ? 128 : TPR;
}

template <typename T, bool RES, int TPR>
__global__ void __launch_bounds__(generic_threads<TPR>()) rms_generic_kernel(const RmsArgs a) {
    constexpr int VEC = 16 / sizeof(T);
    constexpr int ROWS = generic_threads<TPR>() / TPR;
    using P = Packed<T, VEC>;
    __shared__ float scratch[TPR / 32];
    pdl_enter();
    const int64_t row = static_cast<int64_t>(blockIdx.x) * ROWS + threadIdx.x / TPR;
    const int lane = static_cast<int>(threadIdx.x % TPR);
    // A warp whose row is past the end leaves: with a warp per row the
    // reduction is shuffles only, and one-row CTAs have no such warps.
    if (ROWS > 1 && row >= a.rows) return;
    const T* xr = static_cast<const T*>(a.x) + row * a.sx;
    const T* rr = RES ? static_cast<const T*>(a.r) + row * a.sr : nullptr;
    T* ro = RES ? static_cast<T*>(a.ro) + row * a.sro : nullptr;
    T* yr = static_cast<T*>(a.y) + row * a.sy;

    // The row splits into a scalar head, a body of 16-byte vectors and a
    // scalar tail when all of its row pointers sit at the same offset within
    // 16 bytes (ragged widths, e.g. 8200-byte rows); otherwise it is all head.
    const uintptr_t mis = reinterpret_cast<uintptr_t>(xr) & 15u;
    bool same = mis % sizeof(T) == 0 && (reinterpret_cast<uintptr_t>(yr) & 15u) == mis;
    if constexpr (RES)
        same = same && (reinterpret_cast<uintptr_t>(rr) & 15u) == mis && (reinterpret_cast<uintptr_t>(ro) & 15u) == mis;
    int head = same ? static_cast<int>(((16u - mis) & 15u) / sizeof(T)) : a.h;
    if (head > a.h) head = a.h;
    const int nvec = (a.h - head) / VEC;
    const int tail = head + nvec * VEC;

    // Rounded squares: each 16-byte vector's summed pairwise in fp32, those
    // sums and the ends' squares accumulated in fp64 per thread (any row
    // length stays within a few fp32 roundings of the exact sum), then
    // pairwise across threads. One conversion and one fp64 add per vector:
    // per element they made the kernel issue-bound.
    double acc = 0.0;
    auto first_pass = [&](int col) {
        float f = to_f32(xr[col]);
        if constexpr (RES) {
            const T s = from_f32<T>(__fadd_rn(f, to_f32(rr[col])));
            ro[col] = s;
            f = to_f32(s);
        }
        acc += static_cast<double>(__fmul_rn(f, f));
    };
    for (int col = lane; col < head; col += TPR) first_pass(col);
    for (int col = tail + lane; col < a.h; col += TPR) first_pass(col);
    for (int v = lane; v < nvec; v += TPR) {
        const int col = head + v * VEC;
        P xv = ld_stream<T, VEC>(xr + col);
        if constexpr (RES) {
            const P rv = ld_stream<T, VEC>(rr + col);
#pragma unroll
            for (int e = 0; e < VEC; e += 2) {
                const float2 xa = get2<T, VEC>(xv, e);
                const float2 ra = get2<T, VEC>(rv, e);
                put2<T, VEC>(xv, e, __fadd_rn(xa.x, ra.x), __fadd_rn(xa.y, ra.y));
            }
            st_global<T, VEC>(ro + col, xv);
        }
        float sq[VEC];
#pragma unroll
        for (int e = 0; e < VEC; e += 2) {
            const float2 f = get2<T, VEC>(xv, e);
            sq[e] = __fmul_rn(f.x, f.x);
            sq[e + 1] = __fmul_rn(f.y, f.y);
        }
        acc += static_cast<double>(tree_sum<VEC>(sq));
    }
    const float total = block_sum<TPR>(static_cast<float>(acc), scratch);
    const float inv = rms_inv(total, a);

    // The residual pass reads back what this same thread stored above, with
    // ordinary loads so the compiler keeps them after those stores.
    auto second_pass = [&](int col) {
        const float f = RES ? to_f32(ro[col]) : to_f32(xr[col]);
        yr[col] = from_f32<T>(__fmul_rn(__fmul_rn(f, inv), load_weight(a.w, a.wdtype, col)));
    };
    for (int col = lane; col < head; col += TPR) second_pass(col);
    for (int col = tail + lane; col < a.h; col += TPR) second_pass(col);
    // The body's weights: with the row's dtype they are 16 contiguous bytes
    // per vector at a byte offset that is the same for every vector of the
    // row, so they come from two aligned 16-byte loads and a shift chosen
    // once per row; other weights are read element by element.
    const uintptr_t wb = reinterpret_cast<uintptr_t>(a.w) + static_cast<uintptr_t>(head) * sizeof(T);
    if (a.wdtype == dtype_code<T>() && nvec > 0) {
        const uint4* wv = reinterpret_cast<const uint4*>(wb & ~uintptr_t{15});
        switch (static_cast<int>(wb & 15u)) {
            case 0: generic_body_shifted<T, RES, 0, TPR>(a, xr, ro, yr, head, nvec, inv, wv, lane); break;
            case 2: generic_body_shifted<T, RES, 2, TPR>(a, xr, ro, yr, head, nvec, inv, wv, lane); break;
            case 4: generic_body_shifted<T, RES, 4, TPR>(a, xr, ro, yr, head, nvec, inv, wv, lane); break;
            case 6: generic_body_shifted<T, RES, 6, TPR>(a, xr, ro, yr, head, nvec, inv, wv, lane); break;
            case 8: generic_body_shifted<T, RES, 8, TPR>(a, xr, ro, yr, head, nvec, inv, wv, lane); break;
            case 10: generic_body_shifted<T, RES, 10, TPR>(a, xr, ro, yr, head, nvec, inv, wv, lane); break;
            case 12: generic_body_shifted<T, RES, 12, TPR>(a, xr, ro, yr, head, nvec, inv, wv, lane); break;
            default: generic_body_shifted<T, RES, 14, TPR>(a, xr, ro, yr, head, nvec, inv, wv, lane); break;
        }
        return;
    }
    for (int v = lane; v < nvec; v += TPR) {
        const int col = head + v * VEC;
        const P xv = RES ? ld_cached<T, VEC>(ro + col) : ld_cached<T, VEC>(xr + col);
        P o;
#pragma unroll
        for (int e = 0; e < VEC; e += 2) {
            const float2 f = get2<T, VEC>(xv, e);
            put2<T, VEC>(o, e, __fmul_rn(__fmul_rn(f.x, inv), load_weight(a.w, a.wdtype, col + e)),
                         __fmul_rn(__fmul_rn(f.y, inv), load_weight(a.w, a.wdtype, col + e + 1)));
        }
        st_global<T, VEC>(yr + col, o);
    }
}

// Launches `kernel` on `grid` CTAs of `threads`, grouped in clusters of
// `cluster` CTAs along x when cluster > 1.
template <typename Kernel>
int launch_rows_kernel(Kernel kernel, int64_t grid, int threads, int cluster, const RmsArgs& a, cudaStream_t st,
                       const char* name) {
    if (grid > 0x7fffffff) return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: too many rows", name);
    return launch_ex(kernel, dim3(static_cast<unsigned>(grid)), dim3(threads), 0, cluster, st, a, name);
}

#define AKO_RMS_CASE(T, RES, CL, TPR, NV)                                                     \
    case (CL * 65536 + TPR * 16 + NV): {                                                          \
        constexpr int rows_per_cta = RmsShape<TPR>::kRowsPerCta;                                 \
        const int64_t grid = CL > 1 ? a.rows * CL : (a.rows + rows_per_cta - 1) / rows_per_cta;  \
        return launch_rows_kernel(rms_rows_kernel<T, TPR, NV, RES, CL>, grid, RmsShape<TPR>::kThreads, \
                                  CL, a, st, RES ? "rmsnorm_residual" : "rmsnorm");              \
    }

#define AKO_RMS_ALL_CASES(T, RES) \
    AKO_RMS_CASE(T, RES, 1, 32, 1) \
    AKO_RMS_CASE(T, RES, 1, 32, 2) \
    AKO_RMS_CASE(T, RES, 1, 32, 4) \
    AKO_RMS_CASE(T, RES, 1, 32, 8) \
    AKO_RMS_CASE(T, RES, 1, 32, 16) \
    AKO_RMS_CASE(T, RES, 1, 64, 1) \
    AKO_RMS_CASE(T, RES, 1, 64, 2) \
    AKO_RMS_CASE(T, RES, 1, 64, 4) \
    AKO_RMS_CASE(T, RES, 1, 64, 8) \
    AKO_RMS_CASE(T, RES, 1, 64, 16) \
    AKO_RMS_CASE(T, RES, 1, 128, 1) \
    AKO_RMS_CASE(T, RES, 1, 128, 2) \
    AKO_RMS_CASE(T, RES, 1, 128, 4) \
    AKO_RMS_CASE(T, RES, 1, 128, 8) \
    AKO_RMS_CASE(T, RES, 1, 128, 16) \
    AKO_RMS_CASE(T, RES, 1, 256, 1) \
    AKO_RMS_CASE(T, RES, 1, 256, 2) \
    AKO_RMS_CASE(T, RES, 1, 256, 4) \
    AKO_RMS_CASE(T, RES, 1, 256, 8) \
    AKO_RMS_CASE(T, RES, 1, 512, 1) \
    AKO_RMS_CASE(T, RES, 1, 512, 2) \
    AKO_RMS_CASE(T, RES, 1, 512, 4) \
    AKO_RMS_CASE(T, RES, 1, 512, 8) \
    AKO_RMS_CASE(T, RES, 1, 1024, 1) \
    AKO_RMS_CASE(T, RES, 1, 1024, 2) \
    AKO_RMS_CASE(T, RES, 1, 1024, 4) \
    AKO_RMS_CASE(T, RES, 1, 1024, 8) \
    AKO_RMS_CASE(T, RES, 1, 96, 2) \
    AKO_RMS_CASE(T, RES, 1, 96, 4) \
    AKO_RMS_CASE(T, RES, 1, 160, 2) \
    AKO_RMS_CASE(T, RES, 1, 160, 4) \
    AKO_RMS_CASE(T, RES, 1, 192, 2) \
    AKO_RMS_CASE(T, RES, 1, 192, 4) \
    AKO_RMS_CASE(T, RES, 1, 224, 2) \
    AKO_RMS_CASE(T, RES, 1, 224, 4) \
    AKO_RMS_CASE(T, RES, 1, 320, 2) \
    AKO_RMS_CASE(T, RES, 1, 320, 4) \
    AKO_RMS_CASE(T, RES, 1, 384, 2) \
    AKO_RMS_CASE(T, RES, 1, 384, 4) \
    AKO_RMS_CASE(T, RES, 1, 448, 2) \
    AKO_RMS_CASE(T, RES, 1, 448, 4) \
    AKO_RMS_CASE(T, RES, 1, 640, 2) \
    AKO_RMS_CASE(T, RES, 1, 640, 4) \
    AKO_RMS_CASE(T, RES, 1, 768, 2) \
    AKO_RMS_CASE(T, RES, 1, 768, 4) \
    AKO_RMS_CASE(T, RES, 1, 896, 2) \
    AKO_RMS_CASE(T, RES, 1, 896, 4) \
    AKO_RMS_CASE(T, RES, 2, 64, 4) \
    AKO_RMS_CASE(T, RES, 2, 128, 1) \
    AKO_RMS_CASE(T, RES, 2, 128, 2) \
    AKO_RMS_CASE(T, RES, 2, 128, 4) \
    AKO_RMS_CASE(T, RES, 2, 256, 1) \
    AKO_RMS_CASE(T, RES, 2, 256, 2) \
    AKO_RMS_CASE(T, RES, 2, 256, 4) \
    AKO_RMS_CASE(T, RES, 2, 512, 1) \
    AKO_RMS_CASE(T, RES, 2, 512, 2) \
    AKO_RMS_CASE(T, RES, 2, 512, 4) \
    AKO_RMS_CASE(T, RES, 2, 1024, 1) \
    AKO_RMS_CASE(T, RES, 2, 1024, 2) \
    AKO_RMS_CASE(T, RES, 4, 64, 4) \
    AKO_RMS_CASE(T, RES, 4, 128, 1) \
    AKO_RMS_CASE(T, RES, 4, 128, 2) \
    AKO_RMS_CASE(T, RES, 4, 128, 4) \
    AKO_RMS_CASE(T, RES, 4, 256, 1) \
    AKO_RMS_CASE(T, RES, 4, 256, 2) \
    AKO_RMS_CASE(T, RES, 4, 256, 4) \
    AKO_RMS_CASE(T, RES, 4, 512, 1) \
    AKO_RMS_CASE(T, RES, 4, 512, 2) \
    AKO_RMS_CASE(T, RES, 4, 512, 4) \
    AKO_RMS_CASE(T, RES, 4, 1024, 1) \
    AKO_RMS_CASE(T, RES, 4, 1024, 2) \
    AKO_RMS_CASE(T, RES, 8, 64, 4) \
    AKO_RMS_CASE(T, RES, 8, 128, 1) \
    AKO_RMS_CASE(T, RES, 8, 128, 2) \
    AKO_RMS_CASE(T, RES, 8, 128, 4) \
    AKO_RMS_CASE(T, RES, 8, 256, 1) \
    AKO_RMS_CASE(T, RES, 8, 256, 2) \
    AKO_RMS_CASE(T, RES, 8, 256, 4) \
    AKO_RMS_CASE(T, RES, 8, 512, 1) \
    AKO_RMS_CASE(T, RES, 8, 512, 2) \
    AKO_RMS_CASE(T, RES, 8, 512, 4) \
    AKO_RMS_CASE(T, RES, 8, 1024, 1) \
    AKO_RMS_CASE(T, RES, 8, 1024, 2)

// Launches the row-resident kernel for (cluster, tpr, nv); returns -1 when
// that shape is not instantiated.
template <typename T, bool RES>
int launch_rms_rows(const RmsArgs& a, int cluster, int tpr, int nv, cudaStream_t st) {
    switch (cluster * 65536 + tpr * 16 + nv) {
        AKO_RMS_ALL_CASES(T, RES)
        default: return -1;
    }
}

template <typename T, bool RES>
int launch_rms_generic(const RmsArgs& a, int tpr, cudaStream_t st) {
    const char* name = RES ? "rmsnorm_residual(generic)" : "rmsnorm(generic)";
    if (tpr == 32) {
        constexpr int rows = generic_threads<32>() / 32;
        return launch_rows_kernel(rms_generic_kernel<T, RES, 32>, (a.rows + rows - 1) / rows, generic_threads<32>(), 1,
                                  a, st, name);
    }
    return launch_ex(rms_generic_kernel<T, RES, kGenericThreads>, dim3(static_cast<unsigned>(a.rows)),
                     dim3(kGenericThreads), 0, 1, st, a, name);
}

// Polls of a persistent kernel's bounded wait for a bulk copy (about a
// second of polling); when they run out the kernel gives up on its rows.
constexpr uint32_t kWaitPolls = 1u << 24;

// Persistent variant with rows staged in shared memory by bulk copies
// (rmsnorm_tma.cu); -1 when the row is too wide for it.
int launch_rms_staged(const RmsArgs& a, int dtype, bool res, int stages, int ctas_per_sm, uint32_t wait_polls,
                      cudaStream_t st);

// Plain rows of 2049-8192 vectors streamed through shared memory in one or
// two chunks per row (rmsnorm_tma.cu); -1 for other rows.
int launch_rms_chunked(const RmsArgs& a, int dtype, uint32_t wait_polls, cudaStream_t st);

// Host-side shapes of the two persistent kernels (no launch): the staged
// kernel's threads and vectors per thread (false when it does not take the
// row), and the chunked kernel's chunks per row (0 when it does not).
bool rms_staged_shape(int h, int es, bool res, int stages, int ctas_per_sm, int* threads_out, int* nv_out);
int rms_chunks_for(int h, int es);

// Instantiated once per dtype in rmsnorm_{f32,f16,bf16}.cu (compiled in parallel).
#define AKO_RMS_DECLARE(T, KW)                                                        \
    KW template int launch_rms_rows<T, false>(const RmsArgs&, int, int, int, cudaStream_t); \
    KW template int launch_rms_rows<T, true>(const RmsArgs&, int, int, int, cudaStream_t);  \
    KW template int launch_rms_generic<T, false>(const RmsArgs&, int, cudaStream_t);        \
    KW template int launch_rms_generic<T, true>(const RmsArgs&, int, cudaStream_t);

#ifndef AKO_RMS_INSTANTIATING
AKO_RMS_DECLARE(float, extern)
AKO_RMS_DECLARE(__half, extern)
AKO_RMS_DECLARE(__nv_bfloat16, extern)
#endif

}  // namespace ako_b200
