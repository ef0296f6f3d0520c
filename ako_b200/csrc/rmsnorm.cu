// C-ABI entry points for RMSNorm and fused residual-add RMSNorm: argument
// checks, choice of launch shape, dispatch on dtype.
#include <climits>
#include <cmath>

#include "rmsnorm.cuh"

namespace ako_b200 {
namespace {

struct Shape {
    int cluster, tpr, nv;
};

// Launch-shape override ({0, 0, 0}: the built-in table). Measurement builds only.
AKO_B200_OVERRIDE Shape g_override = {0, 0, 0};

// Staging mode: 0 = built-in choice, 1 = row-resident kernel only,
// 2 = staged (bulk-copy ring) kernel where it applies, 3 = chunked kernel
// where it applies (plain rows of 2049-8192 vectors). Measurement builds only.
AKO_B200_OVERRIDE int g_mode = 0;
AKO_B200_OVERRIDE int g_stages = 0;
AKO_B200_OVERRIDE int g_ctas_per_sm = 0;

// Polls of a persistent kernel's bounded wait for a bulk copy (measurement
// builds can lower it to exercise the expiry path).
AKO_B200_OVERRIDE uint32_t g_wait_polls = kWaitPolls;

// Any-width kernel: threads per row (0: the built-in choice below; 32 or 256
// forced). Measurement builds only.
AKO_B200_OVERRIDE int g_generic_tpr = 0;

// Rows of at most this many bytes take the any-width kernel with a warp per
// row (four rows per CTA); wider rows take a 256-thread CTA per row. The
// choice depends on the width alone, so a row's bits do not depend on the
// batch. Measured on B200 (cold L2, 2048-65536 rows): a CTA per row idles
// most of its threads on narrow rows (bf16 1001 wide: 0.25 of peak plain and
// 0.43 fused, against 0.55 and 0.75 with a warp; fp32 517: 0.28 -> 0.70); a
// warp per row is ahead up to 8200-byte plain rows (bf16 4100: 0.69 -> 0.73,
// fp32 2049: 0.64 -> 0.78) and 6000-byte fused ones (bf16 3001: 0.74 ->
// 0.80), and behind above (fused bf16 4100: 0.93 -> 0.76).
constexpr int64_t kGenericWarpMaxBytesPlain = 8704;
constexpr int64_t kGenericWarpMaxBytesFused = 6144;

int generic_tpr(const RmsArgs& a, int es, bool res) {
    if (g_generic_tpr != 0) return g_generic_tpr;
    const int64_t row_bytes = static_cast<int64_t>(a.h) * es;
    return row_bytes <= (res ? kGenericWarpMaxBytesFused : kGenericWarpMaxBytesPlain) ? 32 : kGenericThreads;
}

// Rows from which plain 16-bit rows of 2049-4096 vectors take the staged kernel.
constexpr int64_t kStagedMinRows = 1024;
// Rows from which plain 16-bit rows of 4097-8192 vectors take the chunked
// kernel: fp16 from 148 rows (one per SM) up measured faster; bf16, whose
// row-resident kernel widens by shift and mask, was slower at 148 rows and
// faster from 2048.
constexpr int64_t kChunkedMinRowsF16 = 128;
constexpr int64_t kChunkedMinRowsBF16 = 1024;

// Built-in choice between the row-resident and the staged kernel. Plain
// 16-bit rows of 2049-4096 vectors (16385-32768 elements) need 1024 threads
// x 4 vectors in registers, one CTA per SM, so a row's reduction and stores
// leave HBM idle for that SM; the staged kernel with the same thread layout
// loads the next row into shared memory meanwhile (one stage, one CTA per
// SM): 0.92 against 0.75 of peak at 8192 x 32768 bf16, bit-identical output.
// Below ~1024 rows (7 per SM) the persistent grid's start-up costs about
// what it saves. The chunked kernel with one chunk per row (the row held in
// shared memory instead of registers) measured level with this one. fp32
// and fused rows keep the row-resident kernel, which measured equal or
// faster staged.
bool use_staged(const RmsArgs& a, int es, bool res) {
    if (g_mode == 1 || g_mode == 3) return false;
    if (g_mode == 2) return true;
    const int64_t nvec = static_cast<int64_t>(a.h) * es / 16;
    return g_override.tpr == 0 && !res && es == 2 && nvec > 2048 && nvec <= 4096 && a.rows >= kStagedMinRows;
}

// Built-in choice of the chunked kernel: plain 16-bit rows of 4097-8192
// vectors (32769-65536 elements). The row-resident 1024 x 8 CTA is alone on
// its SM and idles HBM while it reduces and stores a row; the chunked kernel
// streams the next row meanwhile, with the same sums and outputs (8192 x
// 65536: fp16 0.71 -> 0.93 of peak, bf16 0.83 -> 0.90). fp32 rows of that
// many vectors measured level or slower chunked.
bool use_chunked(const RmsArgs& a, int dtype) {
    if (g_mode == 3) return true;
    if (g_mode != 0 || g_override.tpr != 0 || dtype == AKO_B200_F32) return false;
    const int64_t nvec = static_cast<int64_t>(a.h) * 2 / 16;
    const int64_t min_rows = dtype == AKO_B200_F16 ? kChunkedMinRowsF16 : kChunkedMinRowsBF16;
    return nvec > 4096 && nvec <= 8192 && a.rows >= min_rows;
}

// Launch shape for `rows` rows of `nvec` 16-byte vectors, from sweeps of
// every built shape on B200 (bf16, fp16, fp32; 2048..16384 wide; 1 to 32768
// rows; device time per call with the L2 cold, and inside CUDA graphs).
//  * Many rows: one CTA per row. The fused residual form moves two rows in
//    and two out, so two vectors per thread up to 512 threads (1024-vector
//    rows) keep enough loads in flight; wider rows keep 512-1024 threads with
//    4 vectors each. Plain RMSNorm moves half as much per row and wants twice
//    the vectors per thread with fewer threads (64-512 threads x 4, 512 x 8
//    for 4096-vector fp32 rows), which also halves the per-warp fixed work.
//    Fused rows of 4097-8192 vectors are split over a cluster of 8.
//  * Few rows (decode): latency, not bandwidth, decides. One vector per
//    thread (twice the threads) up to 512-vector rows; 2048-vector rows split
//    over a cluster of 4 CTAs and 4096-vector rows over 4 or 8, so a row's
//    loads come from several SMs at once.
// Rows whose vector count is not a power of two (5120 bf16 elements are 640
// vectors) leave up to half of a power-of-two CTA idle. With the table's
// vectors per thread, take the smallest built thread count (multiples of 32
// from 96 to 896) that covers the row, when it is below the table's power of
// two. 5120-wide bf16 rows at 8192
// rows went from 0.86 to 0.94 of peak (fused) and from 0.69 to 0.82 (plain),
// at 32768 rows from 0.98 to 1.07 and from 0.85 to 1.02 (B200, cold L2).
Shape fit_threads(Shape s, int64_t nvec) {
    static const int kFitted[] = {96, 160, 192, 224, 320, 384, 448, 640, 768, 896};
    if (s.cluster != 1 || s.tpr < 128 || (s.nv != 2 && s.nv != 4)) return s;
    const int64_t need = (nvec + s.nv - 1) / s.nv;
    for (int t : kFitted)
        if (t >= need) return t < s.tpr ? Shape{1, t, s.nv} : s;
    return s;
}

// A thread-block cluster splits a row into equal slices of whole 32-vector
// groups, so the fixed summation order sees the same groups as in one CTA.
bool cluster_splits(int64_t nvec, int cluster) { return cluster == 1 || nvec % (32 * cluster) == 0; }

bool pick_shape(int64_t nvec, int64_t rows, bool residual, int es, Shape* out) {
    const Shape& o = g_override;
    if (o.tpr > 0 && static_cast<int64_t>(o.cluster) * o.tpr * o.nv >= nvec && cluster_splits(nvec, o.cluster)) {
        *out = o;
        return true;
    }
    if (rows <= 512 && nvec > 32 && nvec <= 512) {
        if (!residual && nvec > 256 && rows > 64) {
            *out = Shape{1, 256, 2};
            return true;
        }
        // Fused rows move two operands in and two out; from a few hundred rows
        // two vectors per thread (half the threads) beat one. Measured on B200,
        // cold L2, bf16 and fp16, with programmatic launch on (off): 512 rows
        // of 256 vectors 3.78 -> 3.47 us (5.72 -> 4.96), 256 rows of 512
        // vectors 3.88 -> 3.67 (5.73 -> 4.97), 512 rows of 512 5.63 -> 5.22.
        if (residual && nvec > 256 && rows > 128) {
            *out = Shape{1, 256, 2};
            return true;
        }
        if (residual && nvec > 128 && rows > 256) {
            *out = Shape{1, 128, 2};
            return true;
        }
        int tpr = 64;
        while (tpr < nvec) tpr *= 2;
        *out = Shape{1, tpr, 1};
        return true;
    }
    if (nvec > 1024 && nvec <= 2048 && cluster_splits(nvec, 4) && rows <= 64) {
        *out = rows <= 32 ? Shape{4, 512, 1} : Shape{4, 256, 2};
        return true;
    }
    if (nvec > 2048 && nvec <= 4096 && rows <= 64) {
        if (rows <= 8 && cluster_splits(nvec, 8)) {
            *out = Shape{8, 256, 2};
            return true;
        }
        if (cluster_splits(nvec, 4)) {
            *out = Shape{4, 512, 2};
            return true;
        }
    }
    // Narrow rows in bulk: a warp per row (four rows per 128-thread CTA)
    // with 4 or 8 vectors a thread beats a 64-thread CTA per row, whose tiny
    // CTAs cost more to schedule than their rows take to stream. Measured on
    // B200 (bf16, fp16, fp32; 1024-65536 rows): plain rows of 65-128 vectors
    // 0.40-0.55 -> 0.78-0.99 of peak at 65536 rows and better from 4096 rows
    // on; fused rows of 65-112 vectors 0.79-0.93 -> 0.97-0.99 at 65536 rows,
    // better from 16384 (mixed below 8192; 128-vector rows level); plain rows
    // of 129-224 vectors 0.68-0.82 -> 0.74-0.99 at 65536 rows, better from
    // 16384.
    if (nvec > 64 && nvec <= 128 && (!residual || rows >= 8192)) {
        *out = Shape{1, 32, 4};
        return true;
    }
    if (!residual && nvec > 128 && nvec <= 224 && rows >= 16384) {
        *out = Shape{1, 32, 8};
        return true;
    }
    static const Shape fused[] = {{1, 32, 1},  {1, 32, 2},  {1, 64, 2},  {1, 128, 2},
                                  {1, 256, 2}, {1, 512, 2}, {1, 512, 4}, {1, 1024, 4}};
    static const Shape plain[] = {{1, 32, 1},  {1, 32, 2},  {1, 64, 2},  {1, 64, 4},
                                  {1, 128, 4}, {1, 256, 4}, {1, 512, 4}, {1, 512, 8}};
    for (const Shape& s : residual ? fused : plain) {
        if (static_cast<int64_t>(s.tpr) * s.nv >= nvec) {
            // 16-bit rows of 2049-4096 vectors: 512 x 8 needs 106 registers
            // (one CTA per SM); 1024 x 4 streams 11% faster. fp32 keeps 512 x 8.
            if (!residual && es == 2 && s.nv == 8) {
                *out = Shape{1, 1024, 4};
                return true;
            }
            *out = fit_threads(s, nvec);
            return true;
        }
    }
    if (nvec <= 8192) {
        // Rows of 4097-8192 vectors: the fused form splits them over a cluster
        // of 8 CTAs of 256 threads x 4 vectors (0.92 of peak, 0.76 with 512 x 2);
        // plain rows stay in one CTA of 1024 threads x 8 vectors.
        if (residual && cluster_splits(nvec, 8)) {
            *out = Shape{8, 256, 4};
            return true;
        }
        *out = Shape{1, 1024, 8};
        return true;
    }
    return false;
}

// The kernel run() picks for a call, without launching it: kernel 0
// row-resident (cluster x threads x vectors), 1 staged and 2 chunked
// (threads x vectors, cluster 1), 3 any-width.
struct Plan {
    int kernel, cluster, threads, vectors;
};

Plan plan_for(const RmsArgs& a, int dtype, bool res, bool vector_ok) {
    const int es = dtype_size(dtype);
    if (vector_ok && !res && use_chunked(a, dtype)) {
        const int chunks = rms_chunks_for(a.h, es);
        if (chunks > 0) return Plan{2, 1, 1024, 4 * chunks};
    }
    if (vector_ok && use_staged(a, es, res)) {
        const bool chosen = g_mode == 0;
        const int stages = g_stages > 0 ? g_stages : chosen ? 1 : 4;
        const int ctas = g_ctas_per_sm > 0 ? g_ctas_per_sm : chosen ? 1 : 2;
        int threads = 0, nv = 0;
        if (rms_staged_shape(a.h, es, res, stages, ctas, &threads, &nv)) return Plan{1, 1, threads, nv};
    }
    if (vector_ok) {
        Shape s;
        if (pick_shape(a.h / (16 / es), a.rows, res, es, &s)) return Plan{0, s.cluster, s.tpr, s.nv};
    }
    return Plan{3, 1, generic_tpr(a, es, res), 0};
}

template <typename T, bool RES>
int run(const RmsArgs& a, bool vector_ok, cudaStream_t st) {
    if (vector_ok && !RES && use_chunked(a, dtype_code<T>())) {
        const int rc = launch_rms_chunked(a, dtype_code<T>(), g_wait_polls, st);
        if (rc >= 0) return rc;
    }
    if (vector_ok && use_staged(a, sizeof(T), RES)) {
        const int dtype = dtype_code<T>();
        const bool chosen = g_mode == 0;  // the built-in choice above
        const int stages = g_stages > 0 ? g_stages : chosen ? 1 : 4;
        const int ctas = g_ctas_per_sm > 0 ? g_ctas_per_sm : chosen ? 1 : 2;
        const int rc = launch_rms_staged(a, dtype, RES, stages, ctas, g_wait_polls, st);
        if (rc >= 0) return rc;
    }
    if (vector_ok) {
        constexpr int VEC = 16 / sizeof(T);
        Shape s;
        if (pick_shape(a.h / VEC, a.rows, RES, static_cast<int>(sizeof(T)), &s)) {
            const int rc = launch_rms_rows<T, RES>(a, s.cluster, s.tpr, s.nv, st);
            if (rc >= 0) return rc;
        }
    }
    return launch_rms_generic<T, RES>(a, generic_tpr(a, static_cast<int>(sizeof(T)), RES), st);
}

template <bool RES>
int dispatch(const RmsArgs& a, int dtype, bool vector_ok, cudaStream_t st) {
    switch (dtype) {
        case AKO_B200_F32: return run<float, RES>(a, vector_ok, st);
        case AKO_B200_F16: return run<__half, RES>(a, vector_ok, st);
        case AKO_B200_BF16: return run<__nv_bfloat16, RES>(a, vector_ok, st);
        default: return set_error(AKO_B200_ERR_UNSUPPORTED_DTYPE, "unsupported dtype code %d", dtype);
    }
}

// 1 / h for a power of two h (exact in fp32 for h <= 2^126), else 0.
float pow2_reciprocal(int64_t h) {
    return (h & (h - 1)) == 0 ? std::ldexp(1.0f, -std::ilogb(static_cast<double>(h))) : 0.0f;
}

int check_common(const char* op, int64_t rows, int64_t h, int dtype, int wdtype) {
    if (dtype_size(dtype) == 0)
        return set_error(AKO_B200_ERR_UNSUPPORTED_DTYPE, "%s: unsupported dtype code %d", op, dtype);
    if (dtype_size(wdtype) == 0)
        return set_error(AKO_B200_ERR_UNSUPPORTED_DTYPE, "%s: unsupported weight dtype code %d", op, wdtype);
    if (rows < 0) return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: n_rows must be >= 0, got %lld", op,
                                   static_cast<long long>(rows));
    if (h < 1 || h > INT_MAX / 2)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: hidden_dim must be in [1, %d], got %lld", op,
                         INT_MAX / 2, static_cast<long long>(h));
    if (rows > INT_MAX)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: n_rows must be <= %d, got %lld", op, INT_MAX,
                         static_cast<long long>(rows));
    return AKO_B200_OK;
}

int check_operand(const char* op, const char* name, const void* p, int64_t stride, int64_t rows, int64_t h) {
    if (p == nullptr) return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: %s is a null pointer", op, name);
    if (rows > 1 && stride < h)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: %s row stride %lld is smaller than hidden_dim %lld", op,
                         name, static_cast<long long>(stride), static_cast<long long>(h));
    return AKO_B200_OK;
}

}  // namespace
}  // namespace ako_b200

using namespace ako_b200;

extern "C" int ako_b200_rmsnorm(const void* x, int64_t x_row_stride, const void* weight, int weight_dtype, void* y,
                                int64_t y_row_stride, int64_t n_rows, int64_t hidden_dim, double eps, int dtype,
                                void* stream) {
    clear_error();
    const char* op = "ako_b200_rmsnorm";
    int rc = check_common(op, n_rows, hidden_dim, dtype, weight_dtype);
    if (rc) return rc;
    if ((rc = refuse_if_wait_expired(op))) return rc;
    if (n_rows == 0) return AKO_B200_OK;
    if ((rc = check_operand(op, "x", x, x_row_stride, n_rows, hidden_dim))) return rc;
    if ((rc = check_operand(op, "y", y, y_row_stride, n_rows, hidden_dim))) return rc;
    if (weight == nullptr) return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: weight is a null pointer", op);

    RmsArgs a{x, x_row_stride, nullptr, 0, weight, weight_dtype, y, y_row_stride, nullptr, 0,
              n_rows, static_cast<int>(hidden_dim), static_cast<float>(eps), pow2_reciprocal(hidden_dim)};
    const int es = dtype_size(dtype);
    const bool vector_ok = (hidden_dim * es) % 16 == 0 && aligned16(x) && aligned16(y) && aligned16(weight) &&
                           stride_ok16(x_row_stride, n_rows, es) && stride_ok16(y_row_stride, n_rows, es);
    return dispatch<false>(a, dtype, vector_ok, static_cast<cudaStream_t>(stream));
}

extern "C" int ako_b200_rmsnorm_residual(const void* x, int64_t x_row_stride, const void* residual,
                                         int64_t residual_row_stride, const void* weight, int weight_dtype, void* y,
                                         int64_t y_row_stride, void* residual_out, int64_t residual_out_row_stride,
                                         int64_t n_rows, int64_t hidden_dim, double eps, int dtype, void* stream) {
    clear_error();
    const char* op = "ako_b200_rmsnorm_residual";
    int rc = check_common(op, n_rows, hidden_dim, dtype, weight_dtype);
    if (rc) return rc;
    if ((rc = refuse_if_wait_expired(op))) return rc;
    if (n_rows == 0) return AKO_B200_OK;
    if ((rc = check_operand(op, "x", x, x_row_stride, n_rows, hidden_dim))) return rc;
    if ((rc = check_operand(op, "residual", residual, residual_row_stride, n_rows, hidden_dim))) return rc;
    if ((rc = check_operand(op, "y", y, y_row_stride, n_rows, hidden_dim))) return rc;
    if ((rc = check_operand(op, "residual_out", residual_out, residual_out_row_stride, n_rows, hidden_dim)))
        return rc;
    if (weight == nullptr) return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: weight is a null pointer", op);

    RmsArgs a{x,      x_row_stride,  residual, residual_row_stride, weight, weight_dtype,
              y,      y_row_stride,  residual_out, residual_out_row_stride,
              n_rows, static_cast<int>(hidden_dim), static_cast<float>(eps), pow2_reciprocal(hidden_dim)};
    const int es = dtype_size(dtype);
    const bool vector_ok = (hidden_dim * es) % 16 == 0 && aligned16(x) && aligned16(residual) && aligned16(y) &&
                           aligned16(residual_out) && aligned16(weight) && stride_ok16(x_row_stride, n_rows, es) &&
                           stride_ok16(residual_row_stride, n_rows, es) && stride_ok16(y_row_stride, n_rows, es) &&
                           stride_ok16(residual_out_row_stride, n_rows, es);
    return dispatch<true>(a, dtype, vector_ok, static_cast<cudaStream_t>(stream));
}

#ifdef AKO_B200_MEASUREMENT
extern "C" int ako_b200_rmsnorm_set_launch(int cluster, int threads_per_row, int vectors_per_thread) {
    clear_error();
    if (cluster == 0 && threads_per_row == 0 && vectors_per_thread == 0) {
        g_override = {0, 0, 0};
        return AKO_B200_OK;
    }
    static const int single[][2] = {{32, 1},   {32, 2},   {32, 4},   {32, 8},   {32, 16},  {64, 1},  {64, 2},
                                    {64, 4},   {64, 8},   {64, 16},  {128, 1},  {128, 2},  {128, 4}, {128, 8},
                                    {128, 16}, {256, 1},  {256, 2},  {256, 4},  {256, 8},  {512, 1}, {512, 2},
                                    {512, 4},  {512, 8},  {1024, 1}, {1024, 2}, {1024, 4}, {1024, 8}, {96, 2},
                                    {96, 4},   {160, 2},  {160, 4},  {192, 2},  {192, 4},  {224, 2}, {224, 4},
                                    {320, 2},  {320, 4},  {384, 2},  {384, 4},  {448, 2},  {448, 4}, {640, 2},
                                    {640, 4},  {768, 2},  {768, 4},  {896, 2},  {896, 4}};
    static const int split[][2] = {{64, 4},  {128, 1}, {128, 2}, {128, 4}, {256, 1}, {256, 2},
                                   {256, 4}, {512, 1}, {512, 2}, {512, 4}, {1024, 1}, {1024, 2}};
    bool ok = false;
    if (cluster == 1) {
        for (const auto& v : single) ok |= v[0] == threads_per_row && v[1] == vectors_per_thread;
    } else if (cluster == 2 || cluster == 4 || cluster == 8) {
        for (const auto& v : split) ok |= v[0] == threads_per_row && v[1] == vectors_per_thread;
    }
    if (!ok)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "rmsnorm launch shape (cluster %d, %d threads, %d vectors) is not built",
                         cluster, threads_per_row, vectors_per_thread);
    g_override = {cluster, threads_per_row, vectors_per_thread};
    return AKO_B200_OK;
}

extern "C" int ako_b200_rmsnorm_set_generic(int threads_per_row) {
    clear_error();
    if (threads_per_row != 0 && threads_per_row != 32 && threads_per_row != kGenericThreads)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "any-width rmsnorm takes 32 or %d threads per row, got %d",
                         kGenericThreads, threads_per_row);
    g_generic_tpr = threads_per_row;
    return AKO_B200_OK;
}
#endif  // AKO_B200_MEASUREMENT

extern "C" int ako_b200_rmsnorm_plan(int64_t n_rows, int64_t hidden_dim, int dtype, int residual, int aligned,
                                     int* kernel, int* cluster, int* threads_per_row, int* vectors_per_thread) {
    clear_error();
    if (kernel == nullptr || cluster == nullptr || threads_per_row == nullptr || vectors_per_thread == nullptr)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "ako_b200_rmsnorm_plan: null output pointer");
    const int rc = check_common("ako_b200_rmsnorm_plan", n_rows, hidden_dim, dtype, dtype);
    if (rc != AKO_B200_OK) return rc;
    RmsArgs a{};
    a.rows = n_rows;
    a.h = static_cast<int>(hidden_dim);
    const bool vector_ok = aligned != 0 && (hidden_dim * dtype_size(dtype)) % 16 == 0;
    const Plan pl = plan_for(a, dtype, residual != 0, vector_ok);
    *kernel = pl.kernel;
    *cluster = pl.cluster;
    *threads_per_row = pl.threads;
    *vectors_per_thread = pl.vectors;
    return AKO_B200_OK;
}

#ifdef AKO_B200_MEASUREMENT
extern "C" int ako_b200_rmsnorm_set_staging(int mode, int stages, int ctas_per_sm) {
    clear_error();
    if (mode < 0 || mode > 3 || stages < 0 || stages > 8 || ctas_per_sm < 0 || ctas_per_sm > 8)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT,
                         "rmsnorm staging (mode %d, %d stages, %d CTAs per SM) is out of range", mode, stages,
                         ctas_per_sm);
    g_mode = mode;
    g_stages = stages;
    g_ctas_per_sm = ctas_per_sm;
    return AKO_B200_OK;
}

extern "C" unsigned ako_b200_measure_set_wait_polls(unsigned polls) {
    const unsigned prev = g_wait_polls;
    g_wait_polls = polls;
    return prev;
}
#endif  // AKO_B200_MEASUREMENT
