// Shared device helpers for the sm_100a kernels: dtype conversion, 16-byte
// packed accesses with cache hints, and fp32 reductions.
#pragma once

#include <cstdint>
#include <type_traits>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "ako_b200.h"

namespace ako_b200 {

// ------------------------------------------------- programmatic dependent launch
// First statement of every kernel: waits until the previous grid in the
// stream has completed and its writes are visible (returns at once when the
// launch was not programmatic), then lets the next kernel's CTAs be scheduled
// (they wait the same way before touching memory).
__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- conversions
__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
    return __float2bfloat16_rn(v);
}

// The C ABI's dtype code of a storage type.
template <typename T>
constexpr int dtype_code() {
    return std::is_same_v<T, float> ? AKO_B200_F32 : (std::is_same_v<T, __half> ? AKO_B200_F16 : AKO_B200_BF16);
}

// N elements of T moved as one access (16 bytes when N * sizeof(T) == 16).
template <typename T, int N>
struct alignas(sizeof(T) * N) Packed {
    T v[N];
};

// ------------------------------------------------------------ global accesses
// Streaming loads: data read once per launch, one 16-byte access per thread,
// with the default cache policy. Measured on B200, the L1::no_allocate and
// L1::evict_first hints cost 1-5% of bandwidth on row kernels (up to 12% on
// some shapes); the non-coherent path without a hint measures the same as
// this.
template <typename T, int N>
__device__ __forceinline__ Packed<T, N> ld_stream(const T* p) {
    static_assert(sizeof(Packed<T, N>) == 16 || sizeof(Packed<T, N>) <= 8, "pack size");
    Packed<T, N> r;
    if constexpr (sizeof(Packed<T, N>) == 16) {
        uint4 u;
        asm("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(u.x), "=r"(u.y), "=r"(u.z), "=r"(u.w)
                     : "l"(p));
        *reinterpret_cast<uint4*>(&r) = u;
    } else {
        r = *reinterpret_cast<const Packed<T, N>*>(p);
    }
    return r;
}

// Streaming load that bypasses L1 through the non-coherent path. RoPE's
// paired half-row loads run 3-4% faster with it on B200; the row kernels
// run slower (see ld_stream).
template <typename T, int N>
__device__ __forceinline__ Packed<T, N> ld_stream_no_l1(const T* p) {
    static_assert(sizeof(Packed<T, N>) == 16 || sizeof(Packed<T, N>) <= 8, "pack size");
    Packed<T, N> r;
    if constexpr (sizeof(Packed<T, N>) == 16) {
        uint4 u;
        asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
            : "=r"(u.x), "=r"(u.y), "=r"(u.z), "=r"(u.w)
            : "l"(p));
        *reinterpret_cast<uint4*>(&r) = u;
    } else {
        r = *reinterpret_cast<const Packed<T, N>*>(p);
    }
    return r;
}

// Plain cached load (weights and tables that every row or position re-reads).
template <typename T, int N>
__device__ __forceinline__ Packed<T, N> ld_cached(const T* p) {
    return *reinterpret_cast<const Packed<T, N>*>(p);
}

template <typename T, int N>
__device__ __forceinline__ void st_global(T* p, const Packed<T, N>& v) {
    *reinterpret_cast<Packed<T, N>*>(p) = v;
}

// Weight element `i` of a runtime-typed weight vector, as fp32.
__device__ __forceinline__ float load_weight(const void* w, int wdtype, int64_t i) {
    switch (wdtype) {
        case AKO_B200_F16: return __half2float(static_cast<const __half*>(w)[i]);
        case AKO_B200_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(w)[i]);
        default: return static_cast<const float*>(w)[i];
    }
}

// N consecutive weights starting at element `i` (i * sizeof(W) is a multiple
// of N * sizeof(W) rounded down to 16 bytes; the host checks the alignment).
template <int N>
__device__ __forceinline__ void load_weight_vec(const void* w, int wdtype, int64_t i, float (&out)[N]) {
    if (wdtype == AKO_B200_F32) {
        const float* p = static_cast<const float*>(w) + i;
        if constexpr (N % 4 == 0) {
#pragma unroll
            for (int k = 0; k < N; k += 4) {
                const float4 q = *reinterpret_cast<const float4*>(p + k);
                out[k] = q.x; out[k + 1] = q.y; out[k + 2] = q.z; out[k + 3] = q.w;
            }
        } else {
#pragma unroll
            for (int k = 0; k < N; ++k) out[k] = p[k];
        }
    } else if (wdtype == AKO_B200_BF16) {
        const auto q = ld_cached<__nv_bfloat16, N>(static_cast<const __nv_bfloat16*>(w) + i);
        if constexpr (N % 2 == 0) {
#pragma unroll
            for (int k = 0; k < N; k += 2) {
                const uint32_t b = *reinterpret_cast<const uint32_t*>(&q.v[k]);
                out[k] = __uint_as_float(b << 16);
                out[k + 1] = __uint_as_float(b & 0xffff0000u);
            }
        } else {
#pragma unroll
            for (int k = 0; k < N; ++k) out[k] = __bfloat162float(q.v[k]);
        }
    } else {
        const auto q = ld_cached<__half, N>(static_cast<const __half*>(w) + i);
#pragma unroll
        for (int k = 0; k < N; ++k) out[k] = __half2float(q.v[k]);
    }
}


// ------------------------------------------------------------ paired access
// Elements e and e + 1 of a pack as fp32, and back with one rounding each
// (16-bit types convert two at a time: one cvt.rn.{bf16x2,f16x2}.f32). bf16
// widens by moving its bits to the top of the fp32 word (a shift and a mask
// per pair, exact by the format's definition); on B200 that made the RMSNorm
// kernels 1-9% faster than the cvt instruction (get2_cvt keeps the latter).
template <typename T, int N>
__device__ __forceinline__ float2 get2(const Packed<T, N>& p, int e) {
    if constexpr (std::is_same_v<T, float>) {
        return make_float2(p.v[e], p.v[e + 1]);
    } else if constexpr (std::is_same_v<T, __half>) {
        return __half22float2(*reinterpret_cast<const __half2*>(&p.v[e]));
    } else {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(&p.v[e]);
        return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
    }
}

// get2 with the conversion instruction for bf16: SwiGLU, whose ALU pipe is
// the busier one, streams 4% faster with it than with the shift and mask.
template <typename T, int N>
__device__ __forceinline__ float2 get2_cvt(const Packed<T, N>& p, int e) {
    if constexpr (std::is_same_v<T, __nv_bfloat16>) {
        return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&p.v[e]));
    } else {
        return get2<T, N>(p, e);
    }
}

template <typename T, int N>
__device__ __forceinline__ void put2(Packed<T, N>& p, int e, float a, float b) {
    if constexpr (std::is_same_v<T, float>) {
        p.v[e] = a;
        p.v[e + 1] = b;
    } else if constexpr (std::is_same_v<T, __half>) {
        *reinterpret_cast<__half2*>(&p.v[e]) = __floats2half2_rn(a, b);
    } else {
        *reinterpret_cast<__nv_bfloat162*>(&p.v[e]) = __floats2bfloat162_rn(a, b);
    }
}

// ----------------------------------------------------------- integer division
// n / d for 32-bit unsigned n by a divisor fixed at launch, as a multiply-high
// and a shift: Granlund & Montgomery, "Division by Invariant Integers using
// Multiplication" (PLDI 1994), round-up variant with a 64-bit sum, exact for
// every n < 2^32 and 1 <= d < 2^32.
struct FastDiv {
    uint32_t d, mul, shift;

    __host__ static FastDiv make(uint32_t divisor) {
        uint32_t l = 0;
        while ((uint64_t(1) << l) < divisor) ++l;  // ceil(log2(d))
        const uint64_t m = ((uint64_t(1) << 32) * ((uint64_t(1) << l) - divisor)) / divisor + 1;
        return FastDiv{divisor, static_cast<uint32_t>(m), l};
    }

    __device__ __forceinline__ uint32_t div(uint32_t n) const {
        return static_cast<uint32_t>((static_cast<uint64_t>(__umulhi(n, mul)) + n) >> shift);
    }
};

// Starts fetching the L1 line holding element `i` of a runtime-typed weight
// vector, so a later load_weight_vec of it hits L1.
__device__ __forceinline__ void prefetch_weight(const void* w, int wdtype, int64_t i) {
    const char* p = static_cast<const char*>(w) + i * (wdtype == AKO_B200_F32 ? 4 : 2);
    asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}

// ----------------------------------------------------------------- reductions
// Butterfly over `WIDTH` lanes: every lane ends with the bitwise-identical sum
// (fp32 addition is commutative, so partner pairs add the same two values).
template <int WIDTH = 32>
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int off = WIDTH / 2; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off, WIDTH));
    return v;
}

// In-place pairwise sum of N values (pairs at distance 1, 2, 4, ...).
template <int N>
__device__ __forceinline__ float tree_sum(float (&v)[N]) {
#pragma unroll
    for (int s = 1; s < N; s <<= 1) {
#pragma unroll
        for (int i = 0; i + s < N; i += 2 * s) v[i] = __fadd_rn(v[i], v[i + s]);
    }
    return v[0];
}

// ----------------------------------------- fixed-order sums of a row's vectors
// The RMSNorm kernels sum a row's squares in one order that depends only on
// the row width, never on the launch shape or the number of rows:
//   1. each 16-byte vector's squares pairwise (tree_sum<VEC>);
//   2. each group of 32 consecutive vectors by a fold: pairs 16 apart, then
//      8, 4, 2, 1 (what an xor butterfly over the 32 lanes that loaded the
//      group computes, bit for bit in every lane, since fp32 addition is
//      commutative);
//   3. the row's group sums by the same fold over group indices, padded with
//      zeros to a power of two (adding +0 to a sum of squares is exact, so
//      any padding gives the same bits).
// Every launch shape whose thread count per row is a multiple of 32 maps a
// group onto the 32 lanes of one warp: lane l of warp w holds, as its j-th
// vector, vector 32 (j W + w) + l of the row (W warps per row).

constexpr int ilog2_const(int n) { return n <= 1 ? 0 : 1 + ilog2_const(n / 2); }

// Folds each of this lane's NV group partials (p[j]: its vector of group j)
// across the warp. Reduce-scatter: at each of the first log2(NV) levels a lane
// keeps half of its groups and sends the other half to its partner, so the
// warp issues NV - 1 + 5 - log2(NV) shuffles instead of 5 NV. Returns the
// sum of group j = lane >> (5 - log2 NV); lanes with equal top log2(NV) bits
// hold the same bits.
template <int NV>
__device__ __forceinline__ float fold_groups_scatter(float (&p)[NV]) {
    constexpr int L = ilog2_const(NV);
    static_assert((1 << L) == NV && NV <= 32, "NV must be a power of two <= 32");
    const int lane = static_cast<int>(threadIdx.x & 31);
#pragma unroll
    for (int lev = 0; lev < L; ++lev) {
        const int off = 16 >> lev;
        const int n = NV >> (lev + 1);
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < n; ++i) {
            const float send = upper ? p[i] : p[i + n];
            const float keep = upper ? p[i + n] : p[i];
            p[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, off));
        }
    }
    float v = p[0];
#pragma unroll
    for (int off = 16 >> L; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}

// Row sum for a warp that holds a whole row (groups 0..NV-1): the scatter
// leaves group j in lanes whose top log2(NV) bits are j, so folding over
// groups is the butterfly over those bits (offsets 16 down to 32 / NV).
template <int NV>
__device__ __forceinline__ float warp_row_sum(float (&p)[NV]) {
    float v = fold_groups_scatter<NV>(p);
#pragma unroll
    for (int off = 16; off >= (32 >> ilog2_const(NV)); off >>= 1)
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}

// Stores this warp's NV group sums (from fold_groups_scatter) at group index
// j * warps + warp of `gsum`, one lane per group.
template <int NV>
__device__ __forceinline__ void store_group_sums(float v, float* gsum, int warps) {
    constexpr int L = ilog2_const(NV);
    const int lane = static_cast<int>(threadIdx.x & 31);
    if ((lane & ((32 >> L) - 1)) == 0) gsum[(lane >> (5 - L)) * warps + static_cast<int>(threadIdx.x >> 5)] = v;
}

// Fold of `n` group sums (n <= 32 K) read by `load(i)`, in every lane of the
// calling warp: lane l folds its values l + 32 k over k (offsets K/2 .. 1,
// i.e. group offsets 16 K .. 32), then the warp butterflies (16 .. 1).
template <int K, typename Load>
__device__ __forceinline__ float fold_group_sums(int n, Load load) {
    static_assert((K & (K - 1)) == 0, "K must be a power of two");
    const int lane = static_cast<int>(threadIdx.x & 31);
    float v[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
        const int i = lane + 32 * k;
        v[k] = i < n ? load(i) : 0.0f;
    }
#pragma unroll
    for (int off = K / 2; off > 0; off >>= 1) {
#pragma unroll
        for (int i = 0; i < off; ++i) v[i] = __fadd_rn(v[i], v[i + off]);
    }
    return warp_sum(v[0]);
}

// Sum over a CTA of THREADS threads; every thread returns the same value
// (warp partials are combined pairwise in a fixed order). `scratch` holds
// THREADS/32 floats of shared memory and is used once per launch.
template <int THREADS>
__device__ __forceinline__ float block_sum(float v, float* scratch) {
    v = warp_sum(v);
    constexpr int WARPS = THREADS / 32;
    if constexpr (WARPS == 1) {
        return v;
    } else {
        if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = v;
        __syncthreads();
        float p[WARPS];
#pragma unroll
        for (int i = 0; i < WARPS; ++i) p[i] = scratch[i];
        return tree_sum<WARPS>(p);
    }
}


// ------------------------------------------------------- thread-block clusters
__device__ __forceinline__ unsigned cluster_ctarank() {
    unsigned r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Full cluster barrier; orders this CTA's shared-memory writes before other
// CTAs' reads that follow the barrier.
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Reads a float at the same shared-memory offset as `p` in CTA `rank` of
// this cluster (distributed shared memory).
__device__ __forceinline__ float ld_dsmem_f32(const float* p, unsigned rank) {
    const unsigned local = static_cast<unsigned>(__cvta_generic_to_shared(p));
    unsigned remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
    return v;
}


// ------------------------------------------------- bulk copies and mbarriers
// 1-D bulk copies (global -> shared, completed on an mbarrier) for kernels
// that stage rows in shared memory. No multicast form is used anywhere.
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte asynchronous copy from global to shared memory (cp.async, cached in
// L2 only). cp_async_wait_all() waits for this thread's copies; after it, the
// thread reads them (other threads need a barrier as well).
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem)), "l"(gmem) : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Makes initialized mbarriers visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's earlier shared-memory accesses before later bulk copies.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

// Copies `bytes` (a multiple of 16; both addresses 16-byte aligned) from
// global to this CTA's shared memory; completion is counted on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(phase)
        : "memory");
    return done != 0;
}

// Polls `bar` for phase `phase` at most `limit` times (each poll may suspend
// the thread briefly); false when the phase never completed.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t phase, uint32_t limit) {
    for (uint32_t i = 0; i < limit; ++i)
        if (mbar_try_wait(bar, phase)) return true;
    return false;
}

// Status codes that kernels waiting on asynchronous completions record when
// a bounded wait runs out (read and cleared by ako_b200_take_device_status).
constexpr int kStatusWaitTimeout = 1;

}  // namespace ako_b200
