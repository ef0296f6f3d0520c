// Persistent RMSNorm kernels fed by 1-D bulk copies into shared memory
// (cp.async.bulk, mbarrier completion, no multicast), for rows whose
// row-resident CTA sits alone on its SM and leaves HBM idle while it reduces
// and stores a row.
//
// rms_tma_kernel (plain and fused): each CTA owns rows blockIdx.x,
// blockIdx.x + gridDim.x, ... and a ring of `stages` shared-memory slots.
// Thread 0 keeps up to `stages` rows in flight (x, and the residual when
// fused); all threads wait on the slot's mbarrier, read their 16-byte
// vectors into registers, and the slot is refilled with the row `stages`
// ahead as soon as the reduction's barrier shows every thread has read it.
// Arithmetic, rounding and the fixed summation order are those of
// rms_rows_kernel, so outputs are bit-identical to it for every thread count.
//
// rms_chunk_kernel (plain): rows streamed in one or two 64 KB chunks that
// stay in shared memory for both passes; see its comment below.
//
// Every wait is bounded: if a copy never completes, the CTA fills the rows
// it has not produced with NaN, records kStatusWaitTimeout in the
// host-mapped status word (after which every entry point refuses until
// ako_b200_take_device_status clears it), waits (bounded) for its other
// copies, and leaves.
#include <climits>

#include "rmsnorm.cuh"

namespace ako_b200 {

namespace {

constexpr int kTmaThreads = 256;       // rows of up to 8 x 256 vectors
constexpr int kTmaWideThreads = 1024;  // rows of up to 8 x 1024 vectors
constexpr int kMaxStages = 8;
constexpr uint32_t kDrainPolls = 1u << 20;

struct TmaArgs {
    RmsArgs a;
    int stages;
    int stage_bytes;  // x row (+ residual row), multiple of 16
    int* status;      // host-mapped status word
    uint32_t wait_polls;
};

// Records a bounded wait's expiry where the host reads it without
// synchronizing (a plain store: every writer stores the same value).
__device__ __forceinline__ void record_wait_expiry(int* status) {
    *reinterpret_cast<volatile int*>(status) = kStatusWaitTimeout;
    __threadfence_system();
}

// Fills output row `row` (and its residual output when RES) with NaN, so a
// row the CTA gives up on never holds stale memory.
template <typename T, bool RES>
__device__ void nan_fill_row(const RmsArgs& a, int64_t row) {
    const T nan = from_f32<T>(__int_as_float(0x7fc00000));
    T* y = static_cast<T*>(a.y) + row * a.sy;
    T* ro = RES ? static_cast<T*>(a.ro) + row * a.sro : nullptr;
    for (int c = static_cast<int>(threadIdx.x); c < a.h; c += static_cast<int>(blockDim.x)) {
        y[c] = nan;
        if constexpr (RES) ro[c] = nan;
    }
}

template <typename T, int NV, bool RES, int THREADS>
__global__ void __launch_bounds__(THREADS) rms_tma_kernel(const TmaArgs t) {
    constexpr int VEC = 16 / sizeof(T);
    constexpr int WARPS = THREADS / 32;
    using P = Packed<T, VEC>;
    constexpr int GROUPS = NV * WARPS;
    constexpr int K = pow2_ceil((GROUPS + 31) / 32);
    extern __shared__ __align__(128) unsigned char ring[];
    __shared__ uint64_t full[kMaxStages];
    __shared__ float gsum[2][GROUPS];
    pdl_enter();
    const RmsArgs& a = t.a;
    const int h = a.h;
    const uint32_t row_bytes = static_cast<uint32_t>(h) * sizeof(T);

    if (threadIdx.x == 0) {
        for (int s = 0; s < t.stages; ++s) mbar_init(&full[s], 1);
        fence_mbar_init();
    }
    __syncthreads();

    auto issue = [&](int slot, int64_t row) {
        unsigned char* dst = ring + static_cast<size_t>(slot) * t.stage_bytes;
        mbar_expect_tx(&full[slot], RES ? 2 * row_bytes : row_bytes);
        bulk_load(dst, static_cast<const T*>(a.x) + row * a.sx, row_bytes, &full[slot]);
        if constexpr (RES) bulk_load(dst + row_bytes, static_cast<const T*>(a.r) + row * a.sr, row_bytes, &full[slot]);
    };

    const int64_t first = blockIdx.x;
    const int64_t step = gridDim.x;
    if (threadIdx.x == 0) {
        for (int s = 0; s < t.stages; ++s) {
            const int64_t row = first + s * step;
            if (row < a.rows) issue(s, row);
        }
    }

    int k = 0;
    for (int64_t row = first; row < a.rows; row += step, ++k) {
        const int slot = k % t.stages;
        const uint32_t phase = static_cast<uint32_t>(k / t.stages) & 1u;
        const bool ok = mbar_wait_bounded(&full[slot], phase, t.wait_polls);
        if (__syncthreads_or(!ok)) {
            for (int64_t r2 = row; r2 < a.rows; r2 += step) nan_fill_row<T, RES>(a, r2);
            if (threadIdx.x == 0) {
                record_wait_expiry(t.status);
                // Let the copies this CTA started land before it exits.
                for (int j = 0; j < t.stages; ++j) {
                    const int64_t r2 = row + j * step;
                    if (r2 < a.rows)
                        mbar_wait_bounded(&full[(k + j) % t.stages],
                                          static_cast<uint32_t>((k + j) / t.stages) & 1u, kDrainPolls);
                }
            }
            return;
        }

        const unsigned char* base = ring + static_cast<size_t>(slot) * t.stage_bytes;
        const T* xs = reinterpret_cast<const T*>(base);
        P v[NV];
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int col = (j * THREADS + threadIdx.x) * VEC;
            if (col < h) v[j] = *reinterpret_cast<const P*>(xs + col);
        }
        if constexpr (RES) {
            const T* rs = reinterpret_cast<const T*>(base + row_bytes);
            T* ro = static_cast<T*>(a.ro) + row * a.sro;
#pragma unroll
            for (int j = 0; j < NV; ++j) {
                const int col = (j * THREADS + threadIdx.x) * VEC;
                if (col < h) {
                    const P rv = *reinterpret_cast<const P*>(rs + col);
#pragma unroll
                    for (int e = 0; e < VEC; e += 2) {
                        const float2 xa = get2<T, VEC>(v[j], e);
                        const float2 ra = get2<T, VEC>(rv, e);
                        put2<T, VEC>(v[j], e, __fadd_rn(xa.x, ra.x), __fadd_rn(xa.y, ra.y));
                    }
                    st_global<T, VEC>(ro + col, v[j]);
                }
            }
        }
        float part[NV];
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int col = (j * THREADS + threadIdx.x) * VEC;
            float sq[VEC];
#pragma unroll
            for (int e = 0; e < VEC; e += 2) {
                const float2 f = get2<T, VEC>(v[j], e);
                sq[e] = __fmul_rn(f.x, f.x);
                sq[e + 1] = __fmul_rn(f.y, f.y);
            }
            part[j] = col < h ? tree_sum<VEC>(sq) : 0.0f;
        }
        // Group sums alternate between two buffers: a warp writes this
        // buffer again two rows on, after the next row's barrier, which every
        // warp reaches only once it has read this row's sums.
        float* gs = gsum[k & 1];
        store_group_sums<NV>(fold_groups_scatter<NV>(part), gs, WARPS);
        __syncthreads();  // every thread has read the slot and published its groups
        if (threadIdx.x == 0) {
            const int64_t next = row + static_cast<int64_t>(t.stages) * step;
            if (next < a.rows) {
                fence_proxy_async_smem();
                issue(slot, next);
            }
        }
        const float total = fold_group_sums<K>(GROUPS, [&](int i) { return gs[i]; });
        const float inv = rms_inv(total, a);
        T* yr = static_cast<T*>(a.y) + row * a.sy;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int col = (j * THREADS + threadIdx.x) * VEC;
            if (col < h) {
                float w[VEC];
                load_weight_vec<VEC>(a.w, a.wdtype, col, w);
                P o;
#pragma unroll
                for (int e = 0; e < VEC; e += 2) {
                    const float2 f = get2<T, VEC>(v[j], e);
                    put2<T, VEC>(o, e, __fmul_rn(__fmul_rn(f.x, inv), w[e]), __fmul_rn(__fmul_rn(f.y, inv), w[e + 1]));
                }
                st_global<T, VEC>(yr + col, o);
            }
        }
    }
}

// Plain RMSNorm of rows of 2049-8192 vectors, CHUNKS = 1 (up to 4096) or 2
// chunks of at most 1024 x 4 vectors (64 KB) per row. Built for the rows of
// 4097-8192 vectors (16-bit rows of 32769-65536 elements, fp32 of
// 16385-32768), whose 1024 threads x 8 vectors do not fit registers next to
// a next-row prefetch. The chunks stream through a ring of kChunkSlots
// shared-memory slots by 1-D bulk copies and stay there: the sum of squares
// reads them once and the output pass a second time, and each slot is
// refilled with the chunk kChunkSlots ahead as soon as its outputs are
// written, so the next row loads while this one is finished. A chunk's
// weights (when they have the row's dtype) are loaded into registers while
// the row's sum is reduced, or while the previous chunk is written. Thread t
// owns vectors t + 1024 j as in rms_rows_kernel<T, 1024, 4 * CHUNKS>, and
// the row's squares are summed in the same fixed order, so the outputs are
// bit-identical to that kernel's.
constexpr int kChunkSlots = 3;
constexpr int kChunkNV = 4;  // vectors per thread per chunk

struct ChunkArgs {
    RmsArgs a;
    int chunk_bytes;  // bytes of a full chunk (1024 x kChunkNV vectors)
    int* status;      // host-mapped status word
    uint32_t wait_polls;
};

template <typename T, int CHUNKS>
__global__ void __launch_bounds__(kTmaWideThreads, 1) rms_chunk_kernel(const ChunkArgs c) {
    constexpr int VEC = 16 / sizeof(T);
    constexpr int THREADS = kTmaWideThreads;
    constexpr int WARPS = THREADS / 32;
    using P = Packed<T, VEC>;
    constexpr int NVR = CHUNKS * kChunkNV;  // vectors per thread per row
    constexpr int GROUPS = NVR * WARPS;
    constexpr int K = pow2_ceil((GROUPS + 31) / 32);
    extern __shared__ __align__(128) unsigned char ring[];
    __shared__ uint64_t full[kChunkSlots];
    __shared__ float gsum[2][GROUPS];
    pdl_enter();
    const RmsArgs& a = c.a;
    const int h = a.h;
    const uint32_t row_bytes = static_cast<uint32_t>(h) * sizeof(T);
    const int64_t first = blockIdx.x;
    const int64_t step = gridDim.x;
    const int64_t my_rows = first < a.rows ? (a.rows - 1 - first) / step + 1 : 0;
    const int64_t n_chunks = CHUNKS * my_rows;
    const bool w_same = a.wdtype == dtype_code<T>();

    if (threadIdx.x == 0) {
        for (int s = 0; s < kChunkSlots; ++s) mbar_init(&full[s], 1);
        fence_mbar_init();
    }
    __syncthreads();

    // Chunk n of this CTA: part n % CHUNKS of its row n / CHUNKS, into slot
    // n % kChunkSlots; the last part takes the rest of the row.
    auto issue = [&](int64_t n) {
        const int64_t row = first + (n / CHUNKS) * step;
        const int part = static_cast<int>(n % CHUNKS);
        const uint32_t off = static_cast<uint32_t>(part) * static_cast<uint32_t>(c.chunk_bytes);
        const uint32_t bytes = part == CHUNKS - 1 ? row_bytes - off : static_cast<uint32_t>(c.chunk_bytes);
        uint64_t* bar = &full[n % kChunkSlots];
        mbar_expect_tx(bar, bytes);
        bulk_load(ring + static_cast<size_t>(n % kChunkSlots) * c.chunk_bytes,
                  reinterpret_cast<const unsigned char*>(static_cast<const T*>(a.x) + row * a.sx) + off, bytes, bar);
    };
    int64_t issued = 0;
    if (threadIdx.x == 0) {
        for (; issued < kChunkSlots && issued < n_chunks; ++issued) issue(issued);
    }
    // Waits for chunk n; on expiry records the status, lets every copy this
    // CTA started land (bounded), and reports false to all threads.
    auto arrive = [&](int64_t n) -> bool {
        const bool ok = mbar_wait_bounded(&full[n % kChunkSlots], static_cast<uint32_t>(n / kChunkSlots) & 1u,
                                          c.wait_polls);
        if (!__syncthreads_or(!ok)) return true;
        if (threadIdx.x == 0) {
            record_wait_expiry(c.status);
            for (int64_t m = n; m < issued; ++m)
                mbar_wait_bounded(&full[m % kChunkSlots], static_cast<uint32_t>(m / kChunkSlots) & 1u, kDrainPolls);
        }
        return false;
    };

    for (int64_t i = 0; i < my_rows; ++i) {
        const int64_t row = first + i * step;
        const int64_t n0 = CHUNKS * i;
        float part[NVR];  // vector sums, in the row's vector order q * kChunkNV + j
#pragma unroll
        for (int q = 0; q < CHUNKS; ++q) {
            if (!arrive(n0 + q)) {
                for (int64_t r2 = row; r2 < a.rows; r2 += step) nan_fill_row<T, false>(a, r2);
                return;
            }
            const T* xs = reinterpret_cast<const T*>(ring + static_cast<size_t>((n0 + q) % kChunkSlots) * c.chunk_bytes);
#pragma unroll
            for (int j = 0; j < kChunkNV; ++j) {
                const int v = j * THREADS + threadIdx.x;               // vector within the chunk
                const int col = ((q * kChunkNV + j) * THREADS + threadIdx.x) * VEC;  // element within the row
                part[q * kChunkNV + j] = 0.0f;
                if (col < h) {  // a slot holds only its chunk's bytes
                    float sq[VEC];
                    const P xv = *reinterpret_cast<const P*>(xs + v * VEC);
#pragma unroll
                    for (int e = 0; e < VEC; e += 2) {
                        const float2 f = get2<T, VEC>(xv, e);
                        sq[e] = __fmul_rn(f.x, f.x);
                        sq[e + 1] = __fmul_rn(f.y, f.y);
                    }
                    part[q * kChunkNV + j] = tree_sum<VEC>(sq);
                }
            }
        }
        // Weights of the first chunk, loaded while the row's sum is reduced
        // (when they have the row's dtype; other weights load at use).
        P wpre[kChunkNV];
        auto prefetch_w = [&](int q) {
            if (!w_same) return;
#pragma unroll
            for (int j = 0; j < kChunkNV; ++j) {
                const int col = ((q * kChunkNV + j) * THREADS + threadIdx.x) * VEC;
                if (col < h) wpre[j] = ld_cached<T, VEC>(static_cast<const T*>(a.w) + col);
            }
        };
        prefetch_w(0);
        // Group sums alternate between two buffers (see rms_tma_kernel).
        float* gs = gsum[i & 1];
        store_group_sums<NVR>(fold_groups_scatter<NVR>(part), gs, WARPS);
        __syncthreads();
        const float inv = rms_inv(fold_group_sums<K>(GROUPS, [&](int g) { return gs[g]; }), a);
        T* yr = static_cast<T*>(a.y) + row * a.sy;
#pragma unroll
        for (int q = 0; q < CHUNKS; ++q) {
            const int64_t n = n0 + q;
            const T* xs = reinterpret_cast<const T*>(ring + static_cast<size_t>(n % kChunkSlots) * c.chunk_bytes);
#pragma unroll
            for (int j = 0; j < kChunkNV; ++j) {
                const int v = j * THREADS + threadIdx.x;
                const int col = ((q * kChunkNV + j) * THREADS + threadIdx.x) * VEC;
                if (col < h) {
                    const P xv = *reinterpret_cast<const P*>(xs + v * VEC);
                    float w[VEC];
                    if (w_same) {
#pragma unroll
                        for (int e = 0; e < VEC; e += 2) {
                            const float2 wf = get2<T, VEC>(wpre[j], e);
                            w[e] = wf.x;
                            w[e + 1] = wf.y;
                        }
                    } else {
                        load_weight_vec<VEC>(a.w, a.wdtype, col, w);
                    }
                    P o;
#pragma unroll
                    for (int e = 0; e < VEC; e += 2) {
                        const float2 f = get2<T, VEC>(xv, e);
                        put2<T, VEC>(o, e, __fmul_rn(__fmul_rn(f.x, inv), w[e]),
                                     __fmul_rn(__fmul_rn(f.y, inv), w[e + 1]));
                    }
                    st_global<T, VEC>(yr + col, o);
                }
            }
            if (q + 1 < CHUNKS) prefetch_w(q + 1);
            __syncthreads();  // every thread has read the slot
            if (threadIdx.x == 0 && issued < n_chunks) {
                fence_proxy_async_smem();
                issue(issued);
                ++issued;
            }
        }
    }
}

template <typename T, int CHUNKS>
int launch_chunked(const RmsArgs& a, uint32_t wait_polls, cudaStream_t st) {
    int* status = device_status_word();
    if (status == nullptr) return AKO_B200_ERR_CUDA;
    // One-chunk rows get slots of their own size, which leaves the rest of
    // the SM's shared memory to L1 (the weight stays there).
    const int chunk_bytes = CHUNKS == 1 ? a.h * static_cast<int>(sizeof(T)) : kTmaWideThreads * kChunkNV * 16;
    ChunkArgs c{a, chunk_bytes, status, wait_polls};
    const size_t smem = static_cast<size_t>(kChunkSlots) * chunk_bytes;
    auto kernel = rms_chunk_kernel<T, CHUNKS>;
    // Largest ring already allowed for this instantiation, per device.
    static size_t configured[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
    if (smem > configured[dev]) {
        const cudaError_t e =
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) {
            cudaGetLastError();
            return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "rmsnorm(chunked): %zu bytes of shared memory: %s", smem,
                             cudaGetErrorString(e));
        }
        configured[dev] = smem;
    }
    int64_t grid = sm_count();
    if (grid > a.rows) grid = a.rows;
    return launch_ex(kernel, dim3(static_cast<unsigned>(grid)), dim3(kTmaWideThreads), smem, 1, st, c,
                     "rmsnorm(chunked)");
}

template <typename T, int NV, bool RES, int THREADS>
int launch_one(const RmsArgs& a, int stages, int ctas_per_sm, uint32_t wait_polls, cudaStream_t st) {
    int* status = device_status_word();
    if (status == nullptr) return AKO_B200_ERR_CUDA;
    const int row_bytes = a.h * static_cast<int>(sizeof(T));
    TmaArgs t{a, stages, RES ? 2 * row_bytes : row_bytes, status, wait_polls};
    const size_t smem = static_cast<size_t>(stages) * t.stage_bytes;
    auto kernel = rms_tma_kernel<T, NV, RES, THREADS>;
    // Largest ring already allowed for this instantiation, per device.
    static int configured_bytes[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
    if (static_cast<int>(smem) > configured_bytes[dev]) {
        const cudaError_t e =
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) {
            cudaGetLastError();
            return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "rmsnorm(staged): %zu bytes of shared memory: %s", smem,
                             cudaGetErrorString(e));
        }
        configured_bytes[dev] = static_cast<int>(smem);
    }
    // A persistent grid must be resident all at once: no more CTAs per SM than
    // the registers, threads and shared memory allow.
    int fit = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&fit, kernel, THREADS, smem) != cudaSuccess || fit < 1) {
        cudaGetLastError();
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "rmsnorm(staged): a %d-thread CTA with %zu bytes of shared memory does not fit an SM",
                         THREADS, smem);
    }
    int64_t grid = static_cast<int64_t>(sm_count()) * (ctas_per_sm < fit ? ctas_per_sm : fit);
    if (grid > a.rows) grid = a.rows;
    return launch_ex(kernel, dim3(static_cast<unsigned>(grid)), dim3(THREADS), smem, 1, st, t,
                     RES ? "rmsnorm_residual(staged)" : "rmsnorm(staged)");
}

template <typename T, bool RES>
int launch_dtype(const RmsArgs& a, int threads, int nv, int stages, int ctas_per_sm, uint32_t polls, cudaStream_t st) {
    if (threads == kTmaWideThreads) {
        switch (nv) {
            case 4: return launch_one<T, 4, RES, kTmaWideThreads>(a, stages, ctas_per_sm, polls, st);
            case 8:
                // Two rows of 8192 vectors exceed the ring's 200 KB.
                if constexpr (RES) return -1;
                else return launch_one<T, 8, RES, kTmaWideThreads>(a, stages, ctas_per_sm, polls, st);
            default: return -1;
        }
    }
    switch (nv) {
        case 1: return launch_one<T, 1, RES, kTmaThreads>(a, stages, ctas_per_sm, polls, st);
        case 2: return launch_one<T, 2, RES, kTmaThreads>(a, stages, ctas_per_sm, polls, st);
        case 4: return launch_one<T, 4, RES, kTmaThreads>(a, stages, ctas_per_sm, polls, st);
        case 8: return launch_one<T, 8, RES, kTmaThreads>(a, stages, ctas_per_sm, polls, st);
        default: return -1;
    }
}

}  // namespace

// Staged launch for rows of `h` 16-bit or fp32 elements (16-byte aligned rows,
// h * sizeof(T) a multiple of 16); -1 when the row is too wide for it.
bool rms_staged_shape(int h, int es, bool res, int stages, int ctas_per_sm, int* threads_out, int* nv_out) {
    const int nvec = h * es / 16;
    // 256 threads up to 8 vectors each; wider rows take 1024 threads of 4 or 8.
    int threads = kTmaThreads;
    if (nvec > 8 * kTmaThreads) threads = kTmaWideThreads;
    int nv = threads == kTmaThreads ? 1 : 4;
    while (nv * threads < nvec) nv *= 2;
    if (nv > 8 || stages < 1 || stages > kMaxStages || ctas_per_sm < 1) return false;
    const int row_bytes = h * es;
    if (static_cast<int64_t>(stages) * (res ? 2 : 1) * row_bytes > 200 * 1024) return false;
    *threads_out = threads;
    *nv_out = nv;
    return true;
}

int launch_rms_staged(const RmsArgs& a, int dtype, bool res, int stages, int ctas_per_sm, uint32_t wait_polls,
                      cudaStream_t st) {
    int threads = 0, nv = 0;
    if (!rms_staged_shape(a.h, dtype_size(dtype), res, stages, ctas_per_sm, &threads, &nv)) return -1;
    const uint32_t p = wait_polls;
    switch (dtype) {
        case AKO_B200_F32: return res ? launch_dtype<float, true>(a, threads, nv, stages, ctas_per_sm, p, st)
                                      : launch_dtype<float, false>(a, threads, nv, stages, ctas_per_sm, p, st);
        case AKO_B200_F16: return res ? launch_dtype<__half, true>(a, threads, nv, stages, ctas_per_sm, p, st)
                                      : launch_dtype<__half, false>(a, threads, nv, stages, ctas_per_sm, p, st);
        default: return res ? launch_dtype<__nv_bfloat16, true>(a, threads, nv, stages, ctas_per_sm, p, st)
                            : launch_dtype<__nv_bfloat16, false>(a, threads, nv, stages, ctas_per_sm, p, st);
    }
}

// Chunked launch for plain rows of 2049-8192 16-byte vectors (16-byte aligned
// rows): one chunk per row up to 4096 vectors, two above; -1 for other rows.
int rms_chunks_for(int h, int es) {
    const int64_t nvec = static_cast<int64_t>(h) * es / 16;
    const int64_t per_chunk = static_cast<int64_t>(kTmaWideThreads) * kChunkNV;
    if (nvec <= per_chunk / 2 || nvec > 2 * per_chunk) return 0;
    return nvec > per_chunk ? 2 : 1;
}

int launch_rms_chunked(const RmsArgs& a, int dtype, uint32_t wait_polls, cudaStream_t st) {
    const int chunks = rms_chunks_for(a.h, dtype_size(dtype));
    if (chunks == 0) return -1;
    const bool two = chunks == 2;
    const uint32_t p = wait_polls;
    switch (dtype) {
        case AKO_B200_F32: return two ? launch_chunked<float, 2>(a, p, st) : launch_chunked<float, 1>(a, p, st);
        case AKO_B200_F16: return two ? launch_chunked<__half, 2>(a, p, st) : launch_chunked<__half, 1>(a, p, st);
        default:
            return two ? launch_chunked<__nv_bfloat16, 2>(a, p, st) : launch_chunked<__nv_bfloat16, 1>(a, p, st);
    }
}

}  // namespace ako_b200
