// Rotary position embedding for sm_100a, plus its C-ABI entry point.
//
// Definition (reference ako/ops/rope_ref.py:73-107):
//   neox:        y_lo = x_lo * c - x_hi * s,  y_hi = x_lo * s + x_hi * c
//                with x_lo = x[..., i], x_hi = x[..., i + D/2]
//   interleaved: the same with x_lo = x[..., 2i], x_hi = x[..., 2i + 1]
// Each product and the sum/difference are separate fp32 roundings, as in the
// reference's tensor expression, so the fp32 result is bit-identical to it
// and only the final cast rounds.
//
// Work decomposition: one CTA slice per sequence position (b, s). A thread
// owns a chunk of NP consecutive pairs of the head vector; it loads the NP
// cos/sin values of that chunk once and applies them to every head it
// visits, so the table is read once per position rather than once per head.
// Threads in a warp cover consecutive chunks of consecutive heads, so every
// 16-byte access of a warp falls into full 128-byte segments whatever the
// head stride (the (B, H, S, D) layout passed as a transposed view included).
#include <climits>

#include "common.cuh"
#include "host.hpp"

namespace ako_b200 {
namespace {

struct RopeArgs {
    const void* x;
    int64_t xb, xs, xh;
    const float* cos;
    const float* sin;
    int64_t ts;
    void* y;
    int64_t yb, ys, yh;
    int64_t n_pos;
    FastDiv seq;  // position -> (batch, seq) split
    int heads;
    int half;
    int chunks;  // chunks of NP pairs per head
};

int g_heads_per_thread = 0;  // 0: built-in choice

template <int N>
__device__ __forceinline__ void load_table(const float* p, float (&out)[N]) {
    if constexpr (N % 4 == 0) {
#pragma unroll
        for (int k = 0; k < N; k += 4) {
            const float4 q = *reinterpret_cast<const float4*>(p + k);
            out[k] = q.x; out[k + 1] = q.y; out[k + 2] = q.z; out[k + 3] = q.w;
        }
    } else if constexpr (N == 2) {
        const float2 q = *reinterpret_cast<const float2*>(p);
        out[0] = q.x; out[1] = q.y;
    } else {
#pragma unroll
        for (int k = 0; k < N; ++k) out[k] = p[k];
    }
}

__device__ __forceinline__ float rot_lo(float lo, float hi, float c, float s) {
    return __fsub_rn(__fmul_rn(lo, c), __fmul_rn(hi, s));
}
__device__ __forceinline__ float rot_hi(float lo, float hi, float c, float s) {
    return __fadd_rn(__fmul_rn(lo, s), __fmul_rn(hi, c));
}

// Vector path: thread (x = chunk, y = head group, z = position in the CTA)
// owns NP consecutive pairs of HPT consecutive heads. Its NP cos/sin values
// are loaded once; the 2 * HPT 16-byte loads of its heads are issued before
// any arithmetic.
template <typename T, int NP, bool INTERLEAVED, int HPT>
__global__ void __launch_bounds__(256) rope_vec_kernel(const RopeArgs a) {
    constexpr int E = INTERLEAVED ? 2 * NP : NP;  // elements per 16-byte access
    using P = Packed<T, E>;
    const int64_t pos = static_cast<int64_t>(blockIdx.x) * blockDim.z + threadIdx.z;
    if (pos >= a.n_pos) return;
    const uint32_t b = a.seq.div(static_cast<uint32_t>(pos));
    const int64_t s = static_cast<int64_t>(static_cast<uint32_t>(pos) - b * a.seq.d);
    const int c = threadIdx.x;  // blockDim.x == chunks
    const int p0 = c * NP;
    float cs[NP], sn[NP];
    load_table<NP>(a.cos + s * a.ts + p0, cs);
    load_table<NP>(a.sin + s * a.ts + p0, sn);
    const T* xpos = static_cast<const T*>(a.x) + b * a.xb + s * a.xs;
    T* ypos = static_cast<T*>(a.y) + b * a.yb + s * a.ys;

    for (int h0 = threadIdx.y * HPT; h0 < a.heads; h0 += blockDim.y * HPT) {
        P lo[HPT], hi[HPT];
#pragma unroll
        for (int j = 0; j < HPT; ++j) {
            if (h0 + j < a.heads) {
                const T* xp = xpos + (h0 + j) * a.xh;
                if constexpr (INTERLEAVED) {
                    lo[j] = ld_stream<T, E>(xp + 2 * p0);
                } else {
                    lo[j] = ld_stream<T, E>(xp + p0);
                    hi[j] = ld_stream<T, E>(xp + a.half + p0);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < HPT; ++j) {
            if (h0 + j < a.heads) {
                T* yp = ypos + (h0 + j) * a.yh;
                if constexpr (INTERLEAVED) {
                    P o;
#pragma unroll
                    for (int k = 0; k < NP; ++k) {
                        const float2 v = get2<T, E>(lo[j], 2 * k);
                        put2<T, E>(o, 2 * k, rot_lo(v.x, v.y, cs[k], sn[k]), rot_hi(v.x, v.y, cs[k], sn[k]));
                    }
                    st_global<T, E>(yp + 2 * p0, o);
                } else {
                    P ol, oh;
#pragma unroll
                    for (int k = 0; k < NP; k += 2) {
                        const float2 l = get2<T, E>(lo[j], k);
                        const float2 u = get2<T, E>(hi[j], k);
                        put2<T, E>(ol, k, rot_lo(l.x, u.x, cs[k], sn[k]), rot_lo(l.y, u.y, cs[k + 1], sn[k + 1]));
                        put2<T, E>(oh, k, rot_hi(l.x, u.x, cs[k], sn[k]), rot_hi(l.y, u.y, cs[k + 1], sn[k + 1]));
                    }
                    st_global<T, E>(yp + p0, ol);
                    st_global<T, E>(yp + a.half + p0, oh);
                }
            }
        }
    }
}

// Any alignment and head_dim: one pair per thread, element accesses.
template <typename T, bool INTERLEAVED>
__global__ void __launch_bounds__(256) rope_scalar_kernel(const RopeArgs a) {
    const int64_t pos = static_cast<int64_t>(blockIdx.x) * blockDim.z + threadIdx.z;
    if (pos >= a.n_pos) return;
    const uint32_t b = a.seq.div(static_cast<uint32_t>(pos));
    const int64_t s = static_cast<int64_t>(static_cast<uint32_t>(pos) - b * a.seq.d);
    const T* xpos = static_cast<const T*>(a.x) + b * a.xb + s * a.xs;
    T* ypos = static_cast<T*>(a.y) + b * a.yb + s * a.ys;
    for (int p = threadIdx.x; p < a.half; p += blockDim.x) {
        const float c = a.cos[s * a.ts + p];
        const float sn = a.sin[s * a.ts + p];
        const int il = INTERLEAVED ? 2 * p : p;
        const int ih = INTERLEAVED ? 2 * p + 1 : a.half + p;
        for (int h = threadIdx.y; h < a.heads; h += blockDim.y) {
            const T* xp = xpos + h * a.xh;
            T* yp = ypos + h * a.yh;
            const float lo = to_f32(xp[il]), hi = to_f32(xp[ih]);
            yp[il] = from_f32<T>(rot_lo(lo, hi, c, sn));
            yp[ih] = from_f32<T>(rot_hi(lo, hi, c, sn));
        }
    }
}

// Block shape for `chunks` threads per head row: y covers heads in groups of
// `hpt`, z packs positions so a CTA has about 256 threads.
dim3 rope_block(int chunks, int head_groups, int64_t n_pos) {
    const int bx = chunks < 256 ? chunks : 256;
    int by = 256 / bx;
    if (by < 1) by = 1;
    if (by > head_groups) by = head_groups;
    int bz = 256 / (bx * by);
    if (bz < 1) bz = 1;
    if (bz > n_pos) bz = static_cast<int>(n_pos);
    if (bz > 64) bz = 64;
    return dim3(bx, by, bz);
}

template <typename Kernel>
int launch_rope(Kernel kernel, const RopeArgs& a, dim3 block, cudaStream_t st) {
    const int64_t grid = (a.n_pos + block.z - 1) / block.z;
    if (grid > INT_MAX) return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "ako_b200_rope: too many positions");
    kernel<<<static_cast<unsigned>(grid), block, 0, st>>>(a);
    return check_launch("rope");
}

template <typename T, int NP, bool IL>
int launch_vec(RopeArgs a, int hpt, cudaStream_t st) {
    a.chunks = a.half / NP;
    const int groups = (a.heads + hpt - 1) / hpt;
    const dim3 block = rope_block(a.chunks, groups, a.n_pos);
    switch (hpt) {
        case 1: return launch_rope(rope_vec_kernel<T, NP, IL, 1>, a, block, st);
        case 2: return launch_rope(rope_vec_kernel<T, NP, IL, 2>, a, block, st);
        default: return launch_rope(rope_vec_kernel<T, NP, IL, 4>, a, block, st);
    }
}

template <typename T>
int run(RopeArgs a, bool interleaved, bool vector_ok, cudaStream_t st) {
    constexpr int VEC = 16 / sizeof(T);
    // Heads per thread: several heads share a thread's table values and keep
    // more loads in flight; one head per thread when there are few heads.
    int hpt = g_heads_per_thread > 0 ? g_heads_per_thread : (a.heads >= 16 ? 2 : 1);
    const int chunk_pairs = interleaved ? VEC / 2 : VEC;
    // A CTA holds whole head rows (chunks <= 256 threads along x).
    if (vector_ok && a.half % chunk_pairs == 0 && a.half / chunk_pairs <= 256) {
        if (interleaved) return launch_vec<T, VEC / 2, true>(a, hpt, st);
        return launch_vec<T, VEC, false>(a, hpt, st);
    }
    const int bx = a.half < 256 ? a.half : 256;
    const dim3 block = rope_block(bx, a.heads, a.n_pos);
    if (interleaved) return launch_rope(rope_scalar_kernel<T, true>, a, block, st);
    return launch_rope(rope_scalar_kernel<T, false>, a, block, st);
}

}  // namespace
}  // namespace ako_b200

using namespace ako_b200;

extern "C" int ako_b200_rope(const void* x, int64_t x_stride_b, int64_t x_stride_s, int64_t x_stride_h,
                             const float* cos, const float* sin, int64_t table_row_stride, void* y,
                             int64_t y_stride_b, int64_t y_stride_s, int64_t y_stride_h, int64_t batch,
                             int64_t seq_len, int64_t n_heads, int64_t head_dim, int style, int dtype,
                             void* stream) {
    clear_error();
    const char* op = "ako_b200_rope";
    const int es = dtype_size(dtype);
    if (es == 0) return set_error(AKO_B200_ERR_UNSUPPORTED_DTYPE, "%s: unsupported dtype code %d", op, dtype);
    if (style != AKO_B200_ROPE_NEOX && style != AKO_B200_ROPE_INTERLEAVED)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: unknown style code %d", op, style);
    if (batch < 0 || seq_len < 0 || n_heads < 0)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: negative size", op);
    if (head_dim < 2 || head_dim % 2 != 0 || head_dim > INT_MAX / 2)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: head_dim must be even and >= 2, got %lld", op,
                         static_cast<long long>(head_dim));
    if (seq_len > INT_MAX || n_heads > INT_MAX || batch > INT_MAX || batch * seq_len > static_cast<int64_t>(UINT32_MAX))
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: batch * seq_len must be < 2^32", op);
    if (batch == 0 || seq_len == 0 || n_heads == 0) return AKO_B200_OK;
    if (x == nullptr || y == nullptr || cos == nullptr || sin == nullptr)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: null pointer", op);
    const int64_t half = head_dim / 2;
    if (seq_len > 1 && table_row_stride < half)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: table row stride %lld is smaller than head_dim/2", op,
                         static_cast<long long>(table_row_stride));

    // Strides of axes of extent 1 are never used; zero them so they do not
    // defeat the 16-byte path.
    if (batch == 1) x_stride_b = y_stride_b = 0;
    if (seq_len == 1) x_stride_s = y_stride_s = table_row_stride = 0;
    if (n_heads == 1) x_stride_h = y_stride_h = 0;

    RopeArgs a{x,          x_stride_b, x_stride_s, x_stride_h, cos, sin, table_row_stride, y, y_stride_b, y_stride_s,
               y_stride_h, batch * seq_len, FastDiv::make(static_cast<uint32_t>(seq_len)), static_cast<int>(n_heads),
               static_cast<int>(half), 0};
    auto s16 = [&](int64_t st, int elem) { return ((st * elem) & 15) == 0; };
    const bool vector_ok = aligned16(x) && aligned16(y) && aligned16(cos) && aligned16(sin) &&
                           s16(x_stride_b, es) && s16(x_stride_s, es) && s16(x_stride_h, es) &&
                           s16(y_stride_b, es) && s16(y_stride_s, es) && s16(y_stride_h, es) &&
                           s16(table_row_stride, 4) && (half * es) % 16 == 0;
    const bool il = style == AKO_B200_ROPE_INTERLEAVED;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (dtype) {
        case AKO_B200_F32: return run<float>(a, il, vector_ok, st);
        case AKO_B200_F16: return run<__half>(a, il, vector_ok, st);
        default: return run<__nv_bfloat16>(a, il, vector_ok, st);
    }
}

extern "C" int ako_b200_rope_set_launch(int heads_per_thread) {
    clear_error();
    if (heads_per_thread != 0 && heads_per_thread != 1 && heads_per_thread != 2 && heads_per_thread != 4)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "rope heads per thread must be 0, 1, 2 or 4, got %d",
                         heads_per_thread);
    g_heads_per_thread = heads_per_thread;
    return AKO_B200_OK;
}
