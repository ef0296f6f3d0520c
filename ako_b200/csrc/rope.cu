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
    int seq;
    int heads;
    int half;
    int chunks;  // chunks of NP pairs per head
};

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

// NP pairs per thread. VECTOR: the NP (neox) or 2*NP (interleaved) elements
// of a chunk are one 16-byte access; otherwise elements are moved one by one.
template <typename T, int NP, bool INTERLEAVED, bool VECTOR>
__global__ void __launch_bounds__(1024) rope_kernel(const RopeArgs a) {
    const int64_t pos = static_cast<int64_t>(blockIdx.x) * blockDim.z + threadIdx.z;
    if (pos >= a.n_pos) return;
    const int64_t b = pos / a.seq;
    const int64_t s = pos - b * a.seq;
    const float* crow = a.cos + s * a.ts;
    const float* srow = a.sin + s * a.ts;
    const T* xpos = static_cast<const T*>(a.x) + b * a.xb + s * a.xs;
    T* ypos = static_cast<T*>(a.y) + b * a.yb + s * a.ys;

    for (int c = threadIdx.x; c < a.chunks; c += blockDim.x) {
        const int p0 = c * NP;  // first pair of the chunk
        float cs[NP], sn[NP];
        if constexpr (VECTOR) {
            load_table<NP>(crow + p0, cs);
            load_table<NP>(srow + p0, sn);
        } else {
#pragma unroll
            for (int k = 0; k < NP; ++k) { cs[k] = crow[p0 + k]; sn[k] = srow[p0 + k]; }
        }

        for (int h = threadIdx.y; h < a.heads; h += blockDim.y) {
            const T* xp = xpos + h * a.xh;
            T* yp = ypos + h * a.yh;
            float lo[NP], hi[NP];
            if constexpr (!INTERLEAVED) {
                if constexpr (VECTOR) {
                    const auto l = ld_stream<T, NP>(xp + p0);
                    const auto u = ld_stream<T, NP>(xp + a.half + p0);
#pragma unroll
                    for (int k = 0; k < NP; ++k) { lo[k] = to_f32(l.v[k]); hi[k] = to_f32(u.v[k]); }
                } else {
#pragma unroll
                    for (int k = 0; k < NP; ++k) { lo[k] = to_f32(xp[p0 + k]); hi[k] = to_f32(xp[a.half + p0 + k]); }
                }
            } else {
                if constexpr (VECTOR) {
                    const auto q = ld_stream<T, 2 * NP>(xp + 2 * p0);
#pragma unroll
                    for (int k = 0; k < NP; ++k) { lo[k] = to_f32(q.v[2 * k]); hi[k] = to_f32(q.v[2 * k + 1]); }
                } else {
#pragma unroll
                    for (int k = 0; k < NP; ++k) { lo[k] = to_f32(xp[2 * (p0 + k)]); hi[k] = to_f32(xp[2 * (p0 + k) + 1]); }
                }
            }

            T olo[NP], ohi[NP];
#pragma unroll
            for (int k = 0; k < NP; ++k) {
                olo[k] = from_f32<T>(__fsub_rn(__fmul_rn(lo[k], cs[k]), __fmul_rn(hi[k], sn[k])));
                ohi[k] = from_f32<T>(__fadd_rn(__fmul_rn(lo[k], sn[k]), __fmul_rn(hi[k], cs[k])));
            }

            if constexpr (!INTERLEAVED) {
                if constexpr (VECTOR) {
                    Packed<T, NP> l, u;
#pragma unroll
                    for (int k = 0; k < NP; ++k) { l.v[k] = olo[k]; u.v[k] = ohi[k]; }
                    st_global<T, NP>(yp + p0, l);
                    st_global<T, NP>(yp + a.half + p0, u);
                } else {
#pragma unroll
                    for (int k = 0; k < NP; ++k) { yp[p0 + k] = olo[k]; yp[a.half + p0 + k] = ohi[k]; }
                }
            } else {
                if constexpr (VECTOR) {
                    Packed<T, 2 * NP> q;
#pragma unroll
                    for (int k = 0; k < NP; ++k) { q.v[2 * k] = olo[k]; q.v[2 * k + 1] = ohi[k]; }
                    st_global<T, 2 * NP>(yp + 2 * p0, q);
                } else {
#pragma unroll
                    for (int k = 0; k < NP; ++k) { yp[2 * (p0 + k)] = olo[k]; yp[2 * (p0 + k) + 1] = ohi[k]; }
                }
            }
        }
    }
}

// Block shape: x = chunks of a head (<= 256), y = heads, z = positions, with
// about 256 threads per CTA.
dim3 rope_block(int chunks, int heads, int64_t n_pos) {
    const int bx = chunks < 256 ? chunks : 256;
    int by = 256 / bx;
    if (by < 1) by = 1;
    if (by > heads) by = heads;
    int bz = 256 / (bx * by);
    if (bz < 1) bz = 1;
    if (bz > n_pos) bz = static_cast<int>(n_pos);
    if (bz > 64) bz = 64;
    return dim3(bx, by, bz);
}

template <typename T, int NP, bool IL, bool VEC>
int launch(RopeArgs a, cudaStream_t st) {
    a.chunks = a.half / NP;
    const dim3 block = rope_block(a.chunks, a.heads, a.n_pos);
    const int64_t grid = (a.n_pos + block.z - 1) / block.z;
    if (grid > INT_MAX) return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "ako_b200_rope: too many positions");
    rope_kernel<T, NP, IL, VEC><<<static_cast<unsigned>(grid), block, 0, st>>>(a);
    return check_launch("rope");
}

template <typename T>
int run(const RopeArgs& a, bool interleaved, bool vector_ok, cudaStream_t st) {
    constexpr int VEC = 16 / sizeof(T);
    if (!interleaved) {
        if (vector_ok && a.half % VEC == 0) return launch<T, VEC, false, true>(a, st);
        return launch<T, 1, false, false>(a, st);
    }
    if (vector_ok && a.half % (VEC / 2) == 0) return launch<T, VEC / 2, true, true>(a, st);
    return launch<T, 1, true, false>(a, st);
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
    if (seq_len > INT_MAX || n_heads > INT_MAX)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: seq_len and n_heads must fit in int32", op);
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

    RopeArgs a{x,  x_stride_b, x_stride_s, x_stride_h, cos, sin, table_row_stride, y, y_stride_b, y_stride_s,
               y_stride_h, batch * seq_len, static_cast<int>(seq_len), static_cast<int>(n_heads),
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
