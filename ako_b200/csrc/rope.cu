// Rotary position embedding for sm_100a, plus its C-ABI entry points
// (ako_b200_rope for one tensor, ako_b200_rope_qk for a query/key pair).
//
// Definition (reference ako/ops/rope_ref.py:73-107):
//   neox:        y_lo = x_lo * c - x_hi * s,  y_hi = x_lo * s + x_hi * c
//                with x_lo = x[..., i], x_hi = x[..., i + D/2]
//   interleaved: the same with x_lo = x[..., 2i], x_hi = x[..., 2i + 1]
// Each product and the sum/difference are separate fp32 roundings, as in the
// reference's tensor expression, so the fp32 result is bit-identical to it
// and only the final cast rounds.
//
// Work decomposition: a CTA slice per sequence position (b, s). A thread owns
// NP pairs of the head vector (neox: NP consecutive pairs; interleaved: two
// 16-byte chunks of NP/2 pairs, a head's thread count apart); it loads their
// NP cos/sin values once and applies them to every head it visits — the
// heads of up to two tensors (q then k for rope_qk), so a q/k pair shares one
// table read and one launch. Threads in a warp cover consecutive chunks of
// consecutive heads, so every 16-byte access of a warp falls in full
// 128-byte segments whatever the head stride (the (B, H, S, D) layout passed
// as a transposed view included).
#include <climits>

#include "common.cuh"
#include "host.hpp"

namespace ako_b200 {
namespace {

// One rotated tensor: input and output views of logical shape (B, S, heads, D).
struct RopeTensor {
    const void* x;
    int64_t xb, xs, xh;
    void* y;
    int64_t yb, ys, yh;
    int heads;
};

struct RopeArgs {
    RopeTensor t0, t1;  // heads [0, t0.heads) are t0's, the next t1.heads are t1's
    const float* cos;
    const float* sin;
    int64_t ts;
    int64_t n_pos;
    FastDiv seq;  // position -> (batch, seq) split
    int half;
};

AKO_B200_OVERRIDE int g_heads_per_thread = 0;  // 0: built-in choice (measurement builds can force 1, 2, 4)

template <int N>
__device__ __forceinline__ void load_table(const float* p, float* out) {
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

// Input and output row of head `h` (counted over both tensors) at (b, s).
template <typename T>
__device__ __forceinline__ void head_rows(const RopeArgs& a, int h, int64_t b, int64_t s, const T*& xp, T*& yp) {
    const bool first = h < a.t0.heads;
    const int64_t lh = first ? h : h - a.t0.heads;
    const T* x = static_cast<const T*>(first ? a.t0.x : a.t1.x);
    T* y = static_cast<T*>(first ? a.t0.y : a.t1.y);
    xp = x + b * (first ? a.t0.xb : a.t1.xb) + s * (first ? a.t0.xs : a.t1.xs) + lh * (first ? a.t0.xh : a.t1.xh);
    yp = y + b * (first ? a.t0.yb : a.t1.yb) + s * (first ? a.t0.ys : a.t1.ys) + lh * (first ? a.t0.yh : a.t1.yh);
}

// Vector path: thread (x = chunk, y = head group, z = position in the CTA)
// owns NP pairs of HPT consecutive heads. Its NP cos/sin values are loaded
// once; the 16-byte loads of all its heads are issued before any arithmetic.
template <typename T, int NP, bool INTERLEAVED, int HPT>
__global__ void __launch_bounds__(256) rope_vec_kernel(const RopeArgs a) {
    constexpr int E = NP;  // elements per 16-byte access
    using P = Packed<T, E>;
    pdl_enter();
    const int64_t pos = static_cast<int64_t>(blockIdx.x) * blockDim.z + threadIdx.z;
    if (pos >= a.n_pos) return;
    const uint32_t b = a.seq.div(static_cast<uint32_t>(pos));
    const int64_t s = static_cast<int64_t>(static_cast<uint32_t>(pos) - b * a.seq.d);
    // neox: pairs [p0, p0 + NP) of both halves. interleaved: the 16-byte
    // chunks threadIdx.x and threadIdx.x + blockDim.x of the row (NP/2 pairs
    // each), so each warp access covers whole 128-byte lines.
    const int p0 = threadIdx.x * NP;  // blockDim.x == threads per head
    constexpr int Q = NP / 2;         // pairs per interleaved chunk
    const int c0 = threadIdx.x * E, c1 = (threadIdx.x + blockDim.x) * E;  // interleaved element offsets
    float cs[NP], sn[NP];
    if constexpr (INTERLEAVED) {
        load_table<Q>(a.cos + s * a.ts + c0 / 2, cs);
        load_table<Q>(a.cos + s * a.ts + c1 / 2, cs + Q);
        load_table<Q>(a.sin + s * a.ts + c0 / 2, sn);
        load_table<Q>(a.sin + s * a.ts + c1 / 2, sn + Q);
    } else {
        load_table<NP>(a.cos + s * a.ts + p0, cs);
        load_table<NP>(a.sin + s * a.ts + p0, sn);
    }
    const int heads = a.t0.heads + a.t1.heads;

    for (int h0 = threadIdx.y * HPT; h0 < heads; h0 += blockDim.y * HPT) {
        P lo[HPT], hi[HPT];
        T* yrow[HPT];
#pragma unroll
        for (int j = 0; j < HPT; ++j) {
            if (h0 + j < heads) {
                const T* xp;
                head_rows<T>(a, h0 + j, b, s, xp, yrow[j]);
                if constexpr (INTERLEAVED) {
                    lo[j] = ld_stream_no_l1<T, E>(xp + c0);
                    hi[j] = ld_stream_no_l1<T, E>(xp + c1);
                } else {
                    lo[j] = ld_stream_no_l1<T, E>(xp + p0);
                    hi[j] = ld_stream_no_l1<T, E>(xp + a.half + p0);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < HPT; ++j) {
            if (h0 + j < heads) {
                T* yp = yrow[j];
                if constexpr (INTERLEAVED) {
                    P ol, oh;
#pragma unroll
                    for (int k = 0; k < Q; ++k) {
                        const float2 v = get2<T, E>(lo[j], 2 * k);
                        const float2 w = get2<T, E>(hi[j], 2 * k);
                        put2<T, E>(ol, 2 * k, rot_lo(v.x, v.y, cs[k], sn[k]), rot_hi(v.x, v.y, cs[k], sn[k]));
                        put2<T, E>(oh, 2 * k, rot_lo(w.x, w.y, cs[Q + k], sn[Q + k]),
                                   rot_hi(w.x, w.y, cs[Q + k], sn[Q + k]));
                    }
                    st_global<T, E>(yp + c0, ol);
                    st_global<T, E>(yp + c1, oh);
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
    pdl_enter();
    const int64_t pos = static_cast<int64_t>(blockIdx.x) * blockDim.z + threadIdx.z;
    if (pos >= a.n_pos) return;
    const uint32_t b = a.seq.div(static_cast<uint32_t>(pos));
    const int64_t s = static_cast<int64_t>(static_cast<uint32_t>(pos) - b * a.seq.d);
    const int heads = a.t0.heads + a.t1.heads;
    for (int p = threadIdx.x; p < a.half; p += blockDim.x) {
        const float c = a.cos[s * a.ts + p];
        const float sn = a.sin[s * a.ts + p];
        const int il = INTERLEAVED ? 2 * p : p;
        const int ih = INTERLEAVED ? 2 * p + 1 : a.half + p;
        for (int h = threadIdx.y; h < heads; h += blockDim.y) {
            const T* xp;
            T* yp;
            head_rows<T>(a, h, b, s, xp, yp);
            const float lo = to_f32(xp[il]), hi = to_f32(xp[ih]);
            yp[il] = from_f32<T>(rot_lo(lo, hi, c, sn));
            yp[ih] = from_f32<T>(rot_hi(lo, hi, c, sn));
        }
    }
}

// Block shape for `chunks` threads per head row: y covers head groups, z
// packs positions so a CTA has about 256 threads.
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

int launch_rope(void (*kernel)(RopeArgs), const RopeArgs& a, dim3 block, cudaStream_t st, const char* name) {
    const int64_t grid = (a.n_pos + block.z - 1) / block.z;
    if (grid > INT_MAX) return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: too many positions", name);
    return launch_ex(kernel, dim3(static_cast<unsigned>(grid)), block, 0, 1, st, a, name);
}

template <typename T, int NP, bool IL>
int launch_vec(const RopeArgs& a, int hpt, cudaStream_t st, const char* name) {
    const int heads = a.t0.heads + a.t1.heads;
    const dim3 block = rope_block(a.half / NP, (heads + hpt - 1) / hpt, a.n_pos);
    switch (hpt) {
        case 1: return launch_rope(rope_vec_kernel<T, NP, IL, 1>, a, block, st, name);
        case 2: return launch_rope(rope_vec_kernel<T, NP, IL, 2>, a, block, st, name);
        default: return launch_rope(rope_vec_kernel<T, NP, IL, 4>, a, block, st, name);
    }
}

// Heads per thread of the vector kernel (the measurement override, else the
// built-in choice; see run()).
int rope_hpt(bool interleaved) { return g_heads_per_thread > 0 ? g_heads_per_thread : (interleaved ? 2 : 1); }

template <typename T>
int run(const RopeArgs& a, bool interleaved, int access_bytes, cudaStream_t st, const char* name) {
    constexpr int VEC = 16 / sizeof(T);
    const int heads = a.t0.heads + a.t1.heads;
    // Heads per thread, measured on B200 (D = 128, 8..40 heads, 1 to 131072
    // positions): neox is fastest with one (3-4.5% over two at full size,
    // more for decode grids); interleaved with two (17-20% over one), whose
    // four 16-byte accesses per thread then sit a warp width apart.
    const int hpt = rope_hpt(interleaved);
    // A thread rotates NP pairs of a head with two accesses of access_bytes:
    // one in each half (neox) or two chunks a head's thread count apart
    // (interleaved). 16-byte accesses where every operand allows them, else
    // 8 or 4 bytes (at least two elements).
    const int np = access_bytes / static_cast<int>(sizeof(T));
    if (np == VEC) return interleaved ? launch_vec<T, VEC, true>(a, hpt, st, name) : launch_vec<T, VEC, false>(a, hpt, st, name);
    if constexpr (VEC / 2 >= 2) {
        if (np == VEC / 2)
            return interleaved ? launch_vec<T, VEC / 2, true>(a, hpt, st, name)
                               : launch_vec<T, VEC / 2, false>(a, hpt, st, name);
    }
    if constexpr (VEC / 4 >= 2) {
        if (np == VEC / 4)
            return interleaved ? launch_vec<T, VEC / 4, true>(a, hpt, st, name)
                               : launch_vec<T, VEC / 4, false>(a, hpt, st, name);
    }
    const dim3 block = rope_block(a.half < 256 ? a.half : 256, heads, a.n_pos);
    if (interleaved) return launch_rope(rope_scalar_kernel<T, true>, a, block, st, name);
    return launch_rope(rope_scalar_kernel<T, false>, a, block, st, name);
}

struct RopeCall {
    int64_t batch, seq, half;
    int style, dtype;
};

// Checks shared by both entry points; fills the common part of `a`.
int check_call(const char* op, const RopeCall& c, int64_t head_dim, const float* cos, const float* sin,
               int64_t& table_row_stride) {
    if (dtype_size(c.dtype) == 0)
        return set_error(AKO_B200_ERR_UNSUPPORTED_DTYPE, "%s: unsupported dtype code %d", op, c.dtype);
    if (c.style != AKO_B200_ROPE_NEOX && c.style != AKO_B200_ROPE_INTERLEAVED)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: unknown style code %d", op, c.style);
    if (c.batch < 0 || c.seq < 0) return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: negative size", op);
    if (head_dim < 2 || head_dim % 2 != 0 || head_dim > INT_MAX / 2)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: head_dim must be even and >= 2, got %lld", op,
                         static_cast<long long>(head_dim));
    if (c.seq > INT_MAX || c.batch > INT_MAX || c.batch * c.seq > static_cast<int64_t>(UINT32_MAX))
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: batch * seq_len must be < 2^32", op);
    if (c.batch == 0 || c.seq == 0) return AKO_B200_OK;  // nothing to rotate; no pointer is read
    if (cos == nullptr || sin == nullptr)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: null table pointer", op);
    if (c.seq > 1 && table_row_stride < c.half)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: table row stride %lld is smaller than head_dim/2", op,
                         static_cast<long long>(table_row_stride));
    if (c.seq == 1) table_row_stride = 0;
    return AKO_B200_OK;
}

// Builds one tensor's view; strides of extent-1 axes are zeroed so they
// cannot defeat the 16-byte path. Returns false on a null pointer.
bool make_tensor(RopeTensor& t, const void* x, int64_t xb, int64_t xs, int64_t xh, void* y, int64_t yb,
                 int64_t ys, int64_t yh, int64_t heads, const RopeCall& c) {
    if (heads > 0 && (x == nullptr || y == nullptr)) return false;
    if (c.batch == 1) xb = yb = 0;
    if (c.seq == 1) xs = ys = 0;
    if (heads == 1) xh = yh = 0;
    t = RopeTensor{x, xb, xs, xh, y, yb, ys, yh, static_cast<int>(heads)};
    return true;
}

bool aligned_to(const void* p, int bytes) { return (reinterpret_cast<uintptr_t>(p) & (bytes - 1)) == 0; }

// Every access of tensor `t` at `bytes` width starts on a multiple of it.
bool tensor_ok(const RopeTensor& t, int es, int bytes) {
    if (t.heads == 0) return true;
    auto ok = [es, bytes](int64_t st) { return ((st * es) & (bytes - 1)) == 0; };
    return aligned_to(t.x, bytes) && aligned_to(t.y, bytes) && ok(t.xb) && ok(t.xs) && ok(t.xh) && ok(t.yb) &&
           ok(t.ys) && ok(t.yh);
}

// Whether `bytes`-wide accesses (at least two elements) suit the tensors,
// the half head size and the table rows. A thread reads its table values as
// float4 (4+ per group), float2 (2) or floats (1), where a group is its NP
// pairs (neox) or NP/2 (interleaved).
bool access_ok(const RopeArgs& a, int64_t half, int es, bool interleaved, int bytes) {
    const int np = bytes / es;
    if (np < 2 || half % np != 0 || half / np > 256) return false;
    const int group = interleaved ? np / 2 : np;
    const int tb = group >= 4 ? 16 : (group == 2 ? 8 : 4);
    return tensor_ok(a.t0, es, bytes) && tensor_ok(a.t1, es, bytes) && aligned_to(a.cos, tb) &&
           aligned_to(a.sin, tb) && ((a.ts * 4) & (tb - 1)) == 0;
}

// Access width for a call: the widest of 16, 8 and 4 bytes that suits it; 0
// for the scalar kernel. Decode-sized calls (up to 2^15 elements) whose heads
// all fit one pass of a 256-thread CTA with 4-byte accesses take those: each
// thread then rotates one pair per half instead of eight, a shorter chain.
// In CUDA graphs on B200 this took 8-head decode calls (batch 8 and 32, one
// position) from 1.34 to 1.13 and 1.23 us; 32-head calls are slower that way
// (four passes of 8 heads) and keep the widest access.
int access_bytes_for(const RopeArgs& a, int64_t half, int es, bool interleaved) {
    const int heads = a.t0.heads + a.t1.heads;
    const int64_t elems = a.n_pos * heads * half * 2;
    const int np4 = 4 / es;
    if (elems <= (int64_t{1} << 15) && np4 >= 2 && half % np4 == 0 && (half / np4) * heads <= 256 &&
        access_ok(a, half, es, interleaved, 4))
        return 4;
    for (int bytes = 16; bytes >= 4; bytes /= 2)
        if (access_ok(a, half, es, interleaved, bytes)) return bytes;
    return 0;
}

int dispatch(RopeArgs& a, const RopeCall& c, void* stream, const char* name) {
    const int es = dtype_size(c.dtype);
    a.half = static_cast<int>(c.half);
    a.n_pos = c.batch * c.seq;
    a.seq = FastDiv::make(static_cast<uint32_t>(c.seq));
    const bool il = c.style == AKO_B200_ROPE_INTERLEAVED;
    const int bytes = access_bytes_for(a, c.half, es, il);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (c.dtype) {
        case AKO_B200_F32: return run<float>(a, il, bytes, st, name);
        case AKO_B200_F16: return run<__half>(a, il, bytes, st, name);
        default: return run<__nv_bfloat16>(a, il, bytes, st, name);
    }
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
    const RopeCall c{batch, seq_len, head_dim / 2, style, dtype};
    int rc = check_call(op, c, head_dim, cos, sin, table_row_stride);
    if (rc) return rc;
    if ((rc = refuse_if_wait_expired(op))) return rc;
    if (n_heads < 0 || n_heads > INT_MAX) return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: bad n_heads", op);
    if (batch == 0 || seq_len == 0 || n_heads == 0) return AKO_B200_OK;
    RopeArgs a{};
    if (!make_tensor(a.t0, x, x_stride_b, x_stride_s, x_stride_h, y, y_stride_b, y_stride_s, y_stride_h, n_heads, c))
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: null pointer", op);
    a.t1 = RopeTensor{nullptr, 0, 0, 0, nullptr, 0, 0, 0, 0};
    a.cos = cos;
    a.sin = sin;
    a.ts = table_row_stride;
    return dispatch(a, c, stream, "rope");
}

extern "C" int ako_b200_rope_qk(const void* q, int64_t q_stride_b, int64_t q_stride_s, int64_t q_stride_h,
                                const void* k, int64_t k_stride_b, int64_t k_stride_s, int64_t k_stride_h,
                                const float* cos, const float* sin, int64_t table_row_stride, void* q_out,
                                int64_t q_out_stride_b, int64_t q_out_stride_s, int64_t q_out_stride_h, void* k_out,
                                int64_t k_out_stride_b, int64_t k_out_stride_s, int64_t k_out_stride_h,
                                int64_t batch, int64_t seq_len, int64_t q_heads, int64_t k_heads, int64_t head_dim,
                                int style, int dtype, void* stream) {
    clear_error();
    const char* op = "ako_b200_rope_qk";
    const RopeCall c{batch, seq_len, head_dim / 2, style, dtype};
    int rc = check_call(op, c, head_dim, cos, sin, table_row_stride);
    if (rc) return rc;
    if ((rc = refuse_if_wait_expired(op))) return rc;
    if (q_heads < 0 || k_heads < 0 || q_heads + k_heads > INT_MAX)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: bad head counts", op);
    if (batch == 0 || seq_len == 0 || q_heads + k_heads == 0) return AKO_B200_OK;
    RopeArgs a{};
    if (!make_tensor(a.t0, q, q_stride_b, q_stride_s, q_stride_h, q_out, q_out_stride_b, q_out_stride_s,
                     q_out_stride_h, q_heads, c) ||
        !make_tensor(a.t1, k, k_stride_b, k_stride_s, k_stride_h, k_out, k_out_stride_b, k_out_stride_s,
                     k_out_stride_h, k_heads, c))
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: null pointer", op);
    a.cos = cos;
    a.sin = sin;
    a.ts = table_row_stride;
    return dispatch(a, c, stream, "rope_qk");
}

extern "C" int ako_b200_rope_plan(int64_t batch, int64_t seq_len, int64_t n_heads, int64_t head_dim, int style,
                                  int dtype, int* access_bytes, int* heads_per_thread, int* block_x, int* block_y,
                                  int* block_z) {
    clear_error();
    const char* op = "ako_b200_rope_plan";
    if (access_bytes == nullptr || heads_per_thread == nullptr || block_x == nullptr || block_y == nullptr ||
        block_z == nullptr)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: null output pointer", op);
    const int es = dtype_size(dtype);
    if (es == 0) return set_error(AKO_B200_ERR_UNSUPPORTED_DTYPE, "%s: unsupported dtype code %d", op, dtype);
    if (batch < 1 || seq_len < 1 || n_heads < 1 || head_dim < 2 || head_dim % 2 != 0 || n_heads > INT_MAX ||
        head_dim > INT_MAX)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: invalid shape", op);
    if (style != AKO_B200_ROPE_NEOX && style != AKO_B200_ROPE_INTERLEAVED)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "%s: unknown style %d", op, style);
    // A contiguous (batch, seq_len, heads, head_dim) tensor and tables at
    // 256-byte aligned addresses, which are only compared, never read.
    RopeArgs a{};
    const uintptr_t base = 256;
    a.t0 = RopeTensor{reinterpret_cast<const void*>(base), seq_len * n_heads * head_dim, n_heads * head_dim, head_dim,
                      reinterpret_cast<void*>(base), seq_len * n_heads * head_dim, n_heads * head_dim, head_dim,
                      static_cast<int>(n_heads)};
    a.t1 = RopeTensor{nullptr, 0, 0, 0, nullptr, 0, 0, 0, 0};
    a.cos = reinterpret_cast<const float*>(base);
    a.sin = reinterpret_cast<const float*>(base);
    a.ts = head_dim / 2;
    a.n_pos = batch * seq_len;
    a.half = static_cast<int>(head_dim / 2);
    const bool il = style == AKO_B200_ROPE_INTERLEAVED;
    const int bytes = access_bytes_for(a, a.half, es, il);
    const int heads = static_cast<int>(n_heads);
    dim3 block;
    int hpt = 1;
    if (bytes > 0) {
        hpt = rope_hpt(il);
        block = rope_block(a.half / (bytes / es), (heads + hpt - 1) / hpt, a.n_pos);
    } else {
        block = rope_block(a.half < 256 ? a.half : 256, heads, a.n_pos);
    }
    *access_bytes = bytes > 0 ? bytes : es;
    *heads_per_thread = hpt;
    *block_x = static_cast<int>(block.x);
    *block_y = static_cast<int>(block.y);
    *block_z = static_cast<int>(block.z);
    return AKO_B200_OK;
}

#ifdef AKO_B200_MEASUREMENT
extern "C" int ako_b200_rope_set_launch(int heads_per_thread) {
    clear_error();
    if (heads_per_thread != 0 && heads_per_thread != 1 && heads_per_thread != 2 && heads_per_thread != 4)
        return set_error(AKO_B200_ERR_INVALID_ARGUMENT, "rope heads per thread must be 0, 1, 2 or 4, got %d",
                         heads_per_thread);
    g_heads_per_thread = heads_per_thread;
    return AKO_B200_OK;
}
#endif  // AKO_B200_MEASUREMENT
