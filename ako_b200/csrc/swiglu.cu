// SwiGLU activation for sm_100a, plus its C-ABI entry point.
//
// Definition (reference ako/ops/swiglu_ref.py:16-32, F.silu on fp32):
//   y = round_T( silu(g) * u ),  silu(g) = g / (1 + exp(-g)),
//   g = float(gate), u = float(up).
// fp32 outputs evaluate exactly that expression with CUDA's expf and IEEE
// division, so they stay within a few fp32 ulp of the reference. 16-bit
// outputs evaluate g * (1 / (1 + exp(-g))) * u with the MUFU exponential and
// reciprocal (__expf, rcp.approx): the fp32 value is then within ~2.5e-6
// relative of the reference's, three orders of magnitude below the spacing
// of the stored bf16 (2^-8) or fp16 (2^-11) result, so the stored value is
// the reference's or, rarely, its neighbour. That cuts the per-element work
// from ~29 to ~10 instructions: the exact form is issue-bound on B200 at
// HBM rate, the cheap one is not.
//
// Element-wise over an (n_rows x hidden_dim) matrix whose three operands have
// independent row strides (the packed [M, 2F] layout is two strided views).
// Work is a flat sequence of 16-byte vectors; a grid of a few CTAs per SM
// strides over it, each thread keeping UNROLL vectors of both inputs in
// flight before it computes. Row and column of a vector come from one
// multiply-high division (FastDiv) when the operands are not dense.
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
    FastDiv row_div;  // divides by per_row (valid when total < 2^32)
};

constexpr int kThreads = 256;  // default CTA size
constexpr int64_t kTinyElements = int64_t{1} << 15;  // up to this many: 4-byte accesses

// Tuning overrides of the CTA size, of the vectors in flight per thread and
// of the grid's thread budget per SM (0: built-in choice). Measurement builds
// only.
AKO_B200_OVERRIDE int g_threads = 0;
AKO_B200_OVERRIDE int g_unroll = 0;
AKO_B200_OVERRIDE int g_threads_per_sm = 0;
// Dynamic shared memory per CTA (unused by the kernel): limits how many CTAs
// an SM holds at once. Measurement builds only.
AKO_B200_OVERRIDE int g_smem_bytes = 0;

__device__ __forceinline__ float rcp_approx(float x) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

template <typename T>
__device__ __forceinline__ float silu_mul(float g, float u) {
    if constexpr (std::is_same_v<T, float>) {
        const float s = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
        return __fmul_rn(s, u);
    } else {
        if constexpr (std::is_same_v<T, __nv_bfloat16>) {
            // bf16 keeps fp32's exponent range. For g in about [-88.7, -87.3]
            // 1 + exp(-g) exceeds 2^126, its reciprocal is subnormal and the
            // flush-to-zero reciprocal would return 0 where the reference's
            // quotient is a normal bf16 number. The reciprocal of a quarter of
            // the denominator (formed exactly by one fma) stays normal; the
            // product is scaled back. Costs no measurable time at HBM rate,
            // unlike the non-flushing reciprocal (3%). fp16 results that small
            // round to zero either way.
            const float q = rcp_approx(fmaf(0.25f, __expf(-g), 0.25f));
            return ((g * q) * 0.25f) * u;
        } else {
            return (g * rcp_approx(1.0f + __expf(-g))) * u;
        }
    }
}

// FLAT: all three operands are dense (row stride == hidden_dim), so vector
// i sits at element i * VEC of each. Otherwise rows come from FastDiv
// (NARROW, total < 2^32) or a 64-bit division. NC: 16-byte loads through the
// non-coherent path without L1 allocation.
template <typename T, int VEC, int UNROLL, bool FLAT, bool NARROW, int THREADS, bool NC = false>
__global__ void __launch_bounds__(THREADS) swiglu_kernel(const SwigluArgs a) {
    pdl_enter();
    using P = Packed<T, VEC>;
    const T* gp = static_cast<const T*>(a.g);
    const T* up = static_cast<const T*>(a.u);
    T* yp = static_cast<T*>(a.y);
    const int64_t step = static_cast<int64_t>(gridDim.x) * THREADS * UNROLL;
    for (int64_t base = static_cast<int64_t>(blockIdx.x) * THREADS * UNROLL + threadIdx.x; base < a.total;
         base += step) {
        P g[UNROLL], u[UNROLL];
        int64_t yo[UNROLL];
#pragma unroll
        for (int k = 0; k < UNROLL; ++k) {
            const int64_t i = base + static_cast<int64_t>(k) * THREADS;
            if (i < a.total) {
                int64_t go, uo;
                if constexpr (FLAT) {
                    go = uo = yo[k] = i * VEC;
                } else {
                    int64_t row, col;
                    if constexpr (NARROW) {
                        const uint32_t r32 = a.row_div.div(static_cast<uint32_t>(i));
                        row = r32;
                        col = static_cast<int64_t>(static_cast<uint32_t>(i) - r32 * a.row_div.d);
                    } else {
                        row = i / a.per_row;
                        col = i - row * a.per_row;
                    }
                    col *= VEC;
                    go = row * a.sg + col;
                    uo = row * a.su + col;
                    yo[k] = row * a.sy + col;
                }
                if constexpr (VEC * sizeof(T) == 16 && NC) {
                    g[k] = ld_stream_no_l1<T, VEC>(gp + go);
                    u[k] = ld_stream_no_l1<T, VEC>(up + uo);
                } else if constexpr (VEC * sizeof(T) == 16) {
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
            const int64_t i = base + static_cast<int64_t>(k) * THREADS;
            if (i < a.total) {
                P o;
                if constexpr (VEC % 2 == 0) {
#pragma unroll
                    for (int e = 0; e < VEC; e += 2) {
                        const float2 gf = get2_cvt<T, VEC>(g[k], e);
                        const float2 uf = get2_cvt<T, VEC>(u[k], e);
                        put2<T, VEC>(o, e, silu_mul<T>(gf.x, uf.x), silu_mul<T>(gf.y, uf.y));
                    }
                } else {
                    o.v[0] = from_f32<T>(silu_mul<T>(to_f32(g[k].v[0]), to_f32(u[k].v[0])));
                }
                st_global<T, VEC>(yp + yo[k], o);
            }
        }
    }
}

// Dynamic shared memory (unused by the kernel) that leaves room for at most
// four CTAs on an SM: 5 x (48 KB + the 1 KB the runtime reserves per CTA)
// exceeds an SM's 228 KB, 4 x 49 KB does not.
constexpr int kFourResidentSmem = 48 * 1024;

// The grid strides over the vectors with at most `threads_per_sm` threads
// per SM (CTAs of THREADS threads); with `four_resident`, at most four CTAs
// of it are on an SM at once (the rest run as those finish).
template <typename T, int VEC, int UNROLL, int THREADS, bool NC = false>
int launch(SwigluArgs a, bool flat, int threads_per_sm, bool four_resident, cudaStream_t st) {
    const int64_t per_cta = static_cast<int64_t>(THREADS) * UNROLL;
    int64_t grid = (a.total + per_cta - 1) / per_cta;
    const int ctas_per_sm = threads_per_sm >= THREADS ? threads_per_sm / THREADS : 1;
    const int64_t cap = static_cast<int64_t>(sm_count()) * ctas_per_sm;
    if (grid > cap) grid = cap;
    const dim3 g(static_cast<unsigned>(grid));
    const int smem = g_smem_bytes > 0 ? g_smem_bytes : four_resident ? kFourResidentSmem : 0;
    if (flat)
        return launch_ex(swiglu_kernel<T, VEC, UNROLL, true, true, THREADS, NC>, g, dim3(THREADS), smem, 1, st, a, "swiglu");
    if (a.total <= static_cast<int64_t>(UINT_MAX)) {
        a.row_div = FastDiv::make(static_cast<uint32_t>(a.per_row));
        return launch_ex(swiglu_kernel<T, VEC, UNROLL, false, true, THREADS, NC>, g, dim3(THREADS), smem, 1, st, a,
                         "swiglu");
    }
    return launch_ex(swiglu_kernel<T, VEC, UNROLL, false, false, THREADS, NC>, g, dim3(THREADS), smem, 1, st, a, "swiglu");
}

// Launch choice for a call: bytes per access (16, 4 for decode-sized
// problems, or the element size when the operands are not 16-byte aligned),
// CTA size and vectors per thread.
struct SwigluPlan {
    int access_bytes, threads, unroll, threads_per_sm;
    bool four_resident;
    bool no_l1;  // 16-byte loads through the non-coherent path, no L1 allocation
};

// Thread budget per SM of the grid-stride grid, built-in: a full SM of
// threads.
constexpr int kThreadsPerSm = 2048;

SwigluPlan swiglu_plan(int64_t rows, int64_t h, int es, bool vector_ok, bool flat) {
    if (vector_ok && g_threads == 0 && rows * h <= kTinyElements) {
        // Decode-sized problems are latency-bound: two elements per thread
        // (4-byte accesses) spread them over four times the threads, which
        // shortens each thread's chain of conversions, exponentials and
        // reciprocals. In CUDA graphs on B200 this is 0.1 us faster per call
        // for fp16 and fp32 rows of 5632-14336 at 1-2 rows and the same for
        // bf16; above 2^15 elements 16-byte accesses are as fast or faster.
        return SwigluPlan{4, 128, 1, kThreadsPerSm, false, false};
    }
    if (vector_ok) {
        // 256-thread CTAs with one vector of each input per thread (32
        // registers, a full SM of threads) are within 1% of the best shape on
        // every cell measured on B200 (F 5632..14336, 2048..16384 rows, bf16
        // and fp16) and up to 10% faster than two vectors per thread, except
        // dense operands of 2^24 vectors and more, which stream 2-4% faster
        // with two. Small problems (decode rows) use 128-thread CTAs, so the
        // few vectors spread over many SMs (measured fastest up to ~64 rows of
        // 5632..14336).
        //
        // Problems of 2^24 vectors and more stream fastest with two vectors
        // per thread. Dense operands then want a full SM's budget of 256-thread
        // CTAs with at most four of them resident (two even passes): measured
        // on B200 at 16384 x 11008 and x 14336, fp16 1-2% faster than one pass
        // of four (218.2 -> 213.5 us at F 14336) and 3-4% faster than five or
        // more resident, bf16 (59 registers: four resident anyway) unchanged.
        // Strided operands (the packed [M, 2F] halves) want one pass of four
        // (1024 threads per SM): 2-3% faster than a full SM of one-vector
        // threads (bf16 16384 x 14336 packed 224.9 -> 218.5 us), and level
        // with two passes of four.
        //
        // Up to 2^22 vectors (operands of up to 64 MB, the problem within about
        // 1.5x the L2), loads that allocate nothing in L1 (ld.global.nc
        // .L1::no_allocate) stream 1-4% faster on every such config-4 cell
        // measured on B200 (2048 rows, F 5632..14336, bf16 and fp16, dense and
        // packed; bf16 dense 2048 x 14336 30.1 -> 28.9 us); from 4096 rows on
        // they cost 5-10%.
        const int64_t total = rows * (h * es / 16);
        const bool small = total < static_cast<int64_t>(sm_count()) * kThreads * 4;
        const bool huge = total >= (int64_t{1} << 24);
        const int threads = g_threads > 0 ? g_threads : (small ? 128 : kThreads);
        const int unroll = g_unroll > 0 ? g_unroll : (huge ? 2 : 1);
        return SwigluPlan{16, threads, unroll,
                          g_threads_per_sm > 0 ? g_threads_per_sm : (huge && !flat ? 1024 : kThreadsPerSm),
                          huge && flat && g_threads == 0 && g_threads_per_sm == 0,
                          !small && total <= (int64_t{1} << 22) && threads == kThreads && unroll == 1};
    }
    return SwigluPlan{es, 256, 4, kThreadsPerSm, false, false};
}

template <typename T, int VEC>
int launch_vec(const SwigluArgs& a, bool flat, const SwigluPlan& p, cudaStream_t st) {
    const int tps = p.threads_per_sm;
    const bool four = p.four_resident;
    switch (p.threads * 16 + p.unroll) {
        case 64 * 16 + 1: return launch<T, VEC, 1, 64>(a, flat, tps, four, st);
        case 64 * 16 + 2: return launch<T, VEC, 2, 64>(a, flat, tps, four, st);
        case 128 * 16 + 1: return launch<T, VEC, 1, 128>(a, flat, tps, four, st);
        case 128 * 16 + 2: return launch<T, VEC, 2, 128>(a, flat, tps, four, st);
        case 256 * 16 + 1:
            return p.no_l1 ? launch<T, VEC, 1, 256, true>(a, flat, tps, four, st)
                           : launch<T, VEC, 1, 256>(a, flat, tps, four, st);
        case 256 * 16 + 4: return launch<T, VEC, 4, 256>(a, flat, tps, four, st);
        default: return launch<T, VEC, 2, 256>(a, flat, tps, four, st);
    }
}

template <typename T>
int run(SwigluArgs a, int64_t rows, int64_t h, bool vector_ok, bool flat, cudaStream_t st) {
    constexpr int VEC = 16 / sizeof(T);
    const SwigluPlan p = swiglu_plan(rows, h, static_cast<int>(sizeof(T)), vector_ok, flat);
    const int per_access = p.access_bytes / static_cast<int>(sizeof(T));
    a.per_row = h / per_access;
    a.total = rows * a.per_row;
    if (!vector_ok) return launch<T, 1, 4, 256>(a, flat, p.threads_per_sm, false, st);
    if (p.access_bytes == 4) return launch<T, 4 / sizeof(T), 1, 128>(a, flat, p.threads_per_sm, false, st);
    return launch_vec<T, VEC>(a, flat, p, st);
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
    if (const int rc = refuse_if_wait_expired(op)) return rc;
    if (n_rows > 1 && (gate_row_stride < hidden_dim || up_row_stride < hidden_dim || y_row_stride < hidden_dim))
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: a row stride is smaller than hidden_dim %lld", op,
                         static_cast<long long>(hidden_dim));
    if (n_rows == 1) gate_row_stride = up_row_stride = y_row_stride = hidden_dim;

    const bool flat = gate_row_stride == hidden_dim && up_row_stride == hidden_dim && y_row_stride == hidden_dim;
    const bool vector_ok = (hidden_dim * es) % 16 == 0 && aligned16(gate) && aligned16(up) && aligned16(y) &&
                           stride_ok16(gate_row_stride, n_rows, es) && stride_ok16(up_row_stride, n_rows, es) &&
                           stride_ok16(y_row_stride, n_rows, es);
    SwigluArgs a{gate, gate_row_stride, up, up_row_stride, y, y_row_stride, 0, 0, FastDiv{1, 1, 0}};
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (dtype) {
        case AKO_B200_F32: return run<float>(a, n_rows, hidden_dim, vector_ok, flat, st);
        case AKO_B200_F16: return run<__half>(a, n_rows, hidden_dim, vector_ok, flat, st);
        default: return run<__nv_bfloat16>(a, n_rows, hidden_dim, vector_ok, flat, st);
    }
}

extern "C" int ako_b200_swiglu_plan(int64_t n_rows, int64_t hidden_dim, int dtype, int aligned, int dense,
                                    int* access_bytes, int* threads, int* vectors_per_thread, int* threads_per_sm) {
    clear_error();
    if (access_bytes == nullptr || threads == nullptr || vectors_per_thread == nullptr || threads_per_sm == nullptr)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "ako_b200_swiglu_plan: null output pointer");
    const int es = dtype_size(dtype);
    if (es == 0) return set_error(AKO_B200_ERR_UNSUPPORTED_DTYPE, "ako_b200_swiglu_plan: unsupported dtype code %d", dtype);
    if (n_rows < 1 || hidden_dim < 1)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "ako_b200_swiglu_plan: empty problem");
    const bool vector_ok = aligned != 0 && (hidden_dim * es) % 16 == 0;
    const SwigluPlan p = swiglu_plan(n_rows, hidden_dim, es, vector_ok, dense != 0);
    *access_bytes = p.access_bytes;
    *threads = p.threads;
    *vectors_per_thread = p.unroll;
    *threads_per_sm = p.threads_per_sm;
    return AKO_B200_OK;
}

#ifdef AKO_B200_MEASUREMENT
extern "C" int ako_b200_swiglu_set_launch(int threads, int vectors_per_thread) {
    clear_error();
    const int key = threads * 16 + vectors_per_thread;
    if (!(threads == 0 && vectors_per_thread == 0) && key != 64 * 16 + 1 && key != 64 * 16 + 2 &&
        key != 128 * 16 + 1 && key != 128 * 16 + 2 && key != 256 * 16 + 1 && key != 256 * 16 + 2 &&
        key != 256 * 16 + 4)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "swiglu launch (%d threads, %d vectors) is not built",
                         threads, vectors_per_thread);
    g_threads = threads;
    g_unroll = vectors_per_thread;
    return AKO_B200_OK;
}

extern "C" int ako_b200_swiglu_set_grid(int threads_per_sm) {
    clear_error();
    if (threads_per_sm != 0 && (threads_per_sm < 64 || threads_per_sm > 8192 || threads_per_sm % 64 != 0))
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT,
                         "swiglu grid budget must be 0 or a multiple of 64 in [64, 8192], got %d", threads_per_sm);
    g_threads_per_sm = threads_per_sm;
    return AKO_B200_OK;
}

extern "C" int ako_b200_swiglu_set_smem(int bytes) {
    clear_error();
    if (bytes < 0 || bytes > 48 * 1024)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "swiglu shared memory must be in [0, 49152], got %d", bytes);
    g_smem_bytes = bytes;
    return AKO_B200_OK;
}
#endif  // AKO_B200_MEASUREMENT
