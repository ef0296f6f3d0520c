/*
 * ako_b200.h — C ABI of the B200 (sm_100a) kernels for AKO's memory-bound
 * inference operators: RMSNorm, fused residual-add RMSNorm, RoPE and SwiGLU.
 *
 * Every entry point takes plain device pointers, element strides and sizes, a
 * dtype code and a CUDA stream passed as `void*` (a `cudaStream_t`; NULL is
 * the legacy default stream), launches asynchronously on that stream, never
 * synchronizes and never allocates device memory. The return value is an
 * `ako_b200_status`; on failure `ako_b200_last_error()` returns a message for
 * the calling thread.
 *
 * Each function replaces one AKO kernel callable (a `KernelFn` in the
 * reference's registry, reference file:line in the comment above it). A host
 * wrapper with the reference's Python signature lives in
 * `ako_b200/kernels.py`; it allocates the outputs with torch and calls these.
 *
 * Numerics follow the reference's PyTorch definitions: 16-bit inputs are
 * upcast to fp32, intermediates are fp32 operations rounded to nearest in
 * the reference's order (no fused multiply-add where the reference rounds
 * between a multiply and an add), and the result is rounded once to the
 * storage dtype. Two documented departures: RMSNorm sums a row's squares in
 * its own fixed order (see ako_b200_rmsnorm), and 16-bit SwiGLU uses the
 * hardware exponential and reciprocal (see ako_b200_swiglu).
 *
 * This header is the product interface. Launch overrides for measurement
 * (forced shapes and kernels, programmatic launch off, wait limits) exist
 * only in the separate measurement build, libako_b200_measure.so, and are
 * declared in ako_b200_measure.h.
 */
#ifndef AKO_B200_H_
#define AKO_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element types of activations and outputs (and of the RMSNorm weight). */
typedef enum {
    AKO_B200_F32 = 0,
    AKO_B200_F16 = 1,
    AKO_B200_BF16 = 2
} ako_b200_dtype;

typedef enum {
    AKO_B200_OK = 0,
    AKO_B200_ERR_INVALID_ARGUMENT = 1, /* shape, stride, pointer or style problem  */
    AKO_B200_ERR_UNSUPPORTED_DTYPE = 2, /* dtype code outside ako_b200_dtype        */
    AKO_B200_ERR_CUDA = 3,              /* the launch itself failed (cudaError_t)   */
    AKO_B200_ERR_WAIT_EXPIRED = 4       /* refused: see ako_b200_take_device_status */
} ako_b200_status;

/* RoPE pairing conventions (reference: ako/ops/rope_ref.py:1-11). */
typedef enum {
    AKO_B200_ROPE_NEOX = 0,        /* pairs (i, i + head_dim/2)  */
    AKO_B200_ROPE_INTERLEAVED = 1  /* pairs (2i, 2i + 1)         */
} ako_b200_rope_style;

/* ABI version of this header; bumped on any signature change. */
#define AKO_B200_ABI_VERSION 4

int ako_b200_abi_version(void);

/* Human-readable name of a status code (static storage). */
const char* ako_b200_status_string(int status);

/* Message describing the last failure on the calling thread ("" if none). */
const char* ako_b200_last_error(void);

/*
 * RMSNorm over the last dimension:
 *   y[m, :] = (x[m, :] * rsqrt(mean(x[m, :]^2) + eps)) * weight
 * computed in fp32 and rounded once to `dtype`.
 *
 * Replaces the `rmsnorm` KernelFn `fn(x, weight, eps)`:
 *   reference ako/ops/rmsnorm_ref.py:8-23 (definition),
 *   ako/ops/rmsnorm_triton.py:139-160 (the GPU candidate it competes with),
 *   ako/ops/rmsnorm.py:29-31 (call site).
 *
 * x, y:       n_rows rows of hidden_dim elements of `dtype`; row m starts at
 *             element m * x_row_stride (y_row_stride); elements are contiguous.
 * weight:     hidden_dim contiguous elements of `weight_dtype` (any of the
 *             three dtypes).
 * n_rows == 0 is a no-op. hidden_dim >= 1. Strides >= hidden_dim when
 * n_rows > 1. Any alignment is accepted; 16-byte aligned rows use 128-bit
 * accesses.
 *
 * Summation order: on rows of whole 16-byte vectors (hidden_dim * element
 * size a multiple of 16, 16-byte aligned pointers and strides) the squares
 * are summed in one fixed order that depends only on hidden_dim: each
 * vector's squares pairwise, each run of 32 consecutive vectors by a fold
 * (pairs 16, 8, 4, 2, 1 apart), then the runs by the same fold. A row's
 * output bits therefore do not depend on n_rows or on which kernel the call
 * picks. Other rows accumulate in fp64 and round once.
 */
int ako_b200_rmsnorm(const void* x, int64_t x_row_stride,
                     const void* weight, int weight_dtype,
                     void* y, int64_t y_row_stride,
                     int64_t n_rows, int64_t hidden_dim,
                     double eps, int dtype, void* stream);

/*
 * Fused residual add + RMSNorm:
 *   residual_out = round_dtype(x + residual)
 *   y            = rmsnorm(residual_out, weight, eps)
 * Both outputs are written; inputs are read once.
 *
 * Replaces the `rmsnorm_residual` KernelFn `fn(x, residual, weight, eps)`
 * returning `(normed, new_residual)`:
 *   reference ako/ops/rmsnorm_ref.py:26-50 (definition),
 *   ako/ops/rmsnorm_triton.py:163-192 (GPU candidate),
 *   ako/ops/rmsnorm.py:54-56 (call site).
 */
int ako_b200_rmsnorm_residual(const void* x, int64_t x_row_stride,
                              const void* residual, int64_t residual_row_stride,
                              const void* weight, int weight_dtype,
                              void* y, int64_t y_row_stride,
                              void* residual_out, int64_t residual_out_row_stride,
                              int64_t n_rows, int64_t hidden_dim,
                              double eps, int dtype, void* stream);

/*
 * Rotary position embedding on x of logical shape (batch, seq_len, n_heads,
 * head_dim) with arbitrary element strides for the first three axes (the last
 * axis is contiguous), so a (batch, n_heads, seq_len, head_dim)-contiguous
 * tensor can be passed as its transposed view without a copy.
 *   neox:        y[..., i]        = x[..., i] * c_i - x[..., i + D/2] * s_i
 *                y[..., i + D/2]  = x[..., i] * s_i + x[..., i + D/2] * c_i
 *   interleaved: the same on pairs (2i, 2i + 1).
 * c_i = cos[s, i], s_i = sin[s, i]: fp32 tables of seq_len rows of head_dim/2
 * contiguous values, row s at element s * table_row_stride (a row slice of a
 * longer table is passed by pointer offset, no copy).
 *
 * Replaces the `rope` KernelFn `fn(x, cos, sin, style)`:
 *   reference ako/ops/rope_ref.py:73-107 (definition), :57-70 (validation),
 *   ako/ops/rope_triton.py:97-156 (GPU candidate),
 *   ako/ops/rope.py:33-42 (call site).
 */
int ako_b200_rope(const void* x, int64_t x_stride_b, int64_t x_stride_s, int64_t x_stride_h,
                  const float* cos, const float* sin, int64_t table_row_stride,
                  void* y, int64_t y_stride_b, int64_t y_stride_s, int64_t y_stride_h,
                  int64_t batch, int64_t seq_len, int64_t n_heads, int64_t head_dim,
                  int style, int dtype, void* stream);

/*
 * RoPE of a query/key pair in one launch: q (batch, seq_len, q_heads,
 * head_dim) and k (batch, seq_len, k_heads, head_dim), each with its own
 * strides, rotated with the same table; each position's cos/sin values are
 * read once for all q_heads + k_heads heads. Same arithmetic as
 * ako_b200_rope, so each output equals what ako_b200_rope gives for that
 * tensor.
 *
 * Replaces the reference's pair of rope calls in `rope_qk`
 * (ako/ops/rope.py:45-58; decoder call site ako/models/decoder.py:174-175).
 */
int ako_b200_rope_qk(const void* q, int64_t q_stride_b, int64_t q_stride_s, int64_t q_stride_h,
                     const void* k, int64_t k_stride_b, int64_t k_stride_s, int64_t k_stride_h,
                     const float* cos, const float* sin, int64_t table_row_stride,
                     void* q_out, int64_t q_out_stride_b, int64_t q_out_stride_s, int64_t q_out_stride_h,
                     void* k_out, int64_t k_out_stride_b, int64_t k_out_stride_s, int64_t k_out_stride_h,
                     int64_t batch, int64_t seq_len, int64_t q_heads, int64_t k_heads, int64_t head_dim,
                     int style, int dtype, void* stream);

/*
 * SwiGLU activation: y = silu(gate) * up = (gate / (1 + exp(-gate))) * up,
 * evaluated in fp32 and rounded once. gate, up and y are n_rows x hidden_dim
 * with independent row strides, so the packed layout (one [M, 2F] buffer whose
 * halves are gate and up) is passed as two strided views without a copy.
 * fp32 uses CUDA's expf and an IEEE division. 16-bit dtypes use the hardware
 * exponential and reciprocal: the fp32 value is within about 2.5e-6
 * (relative) of the reference's, and the rounded output equals the
 * reference's or one of its two neighbours.
 *
 * Replaces the `swiglu` KernelFn `fn(gate, up)`:
 *   reference ako/ops/swiglu_ref.py:16-32 (definition),
 *   ako/ops/swiglu_triton.py:55-81 (GPU candidate),
 *   ako/ops/swiglu.py:22-24 (call site).
 */
int ako_b200_swiglu(const void* gate, int64_t gate_row_stride,
                    const void* up, int64_t up_row_stride,
                    void* y, int64_t y_row_stride,
                    int64_t n_rows, int64_t hidden_dim,
                    int dtype, void* stream);

/*
 * The kernel an RMSNorm call of `n_rows` x `hidden_dim` in `dtype` would run,
 * without launching anything (host only; no GPU needed): *kernel is 0 for the
 * row-resident kernel (a thread-block cluster of *cluster CTAs, each row
 * slice held by *threads_per_row threads with *vectors_per_thread 16-byte
 * vectors), 1 for the staged and 2 for the chunked persistent kernel
 * (threads and vectors per thread; cluster 1), 3 for the any-width kernel
 * (*threads_per_row 32, a warp per row, or 256, a CTA per row).
 * `residual` selects the fused form; `aligned` says whether the call's
 * pointers and row strides are 16-byte aligned. Follows the library's
 * built-in choice (in the measurement build, any override in force). Not
 * part of the reference's interface; it has no counterpart there.
 */
int ako_b200_rmsnorm_plan(int64_t n_rows, int64_t hidden_dim, int dtype, int residual, int aligned,
                          int* kernel, int* cluster, int* threads_per_row, int* vectors_per_thread);

/*
 * Status of the persistent RMSNorm kernels (the staged and chunked kernels,
 * which wait on 1-D bulk copies). Every such wait is bounded (about a
 * second of polling). If one runs out, the kernel writes NaN into each
 * output row it could not produce (y, and residual_out for the fused form),
 * records the event in a status word in host-mapped memory, and exits. From
 * then on every entry point of this library refuses with
 * AKO_B200_ERR_WAIT_EXPIRED, before launching anything, so the expiry
 * surfaces at the next call without any synchronization on the hot path.
 * This function synchronizes the current device, stores the status in
 * *status (0: no expiry; 1: a wait ran out) and clears it, after which calls
 * are accepted again. Not part of the reference's interface; it has no
 * counterpart there.
 */
int ako_b200_take_device_status(int* status);

/*
 * The launch a RoPE call on contiguous (batch, seq_len, n_heads, head_dim)
 * tensors and tables would get, without launching anything (host only; no
 * GPU needed): bytes per access of x (16, 8 or 4; the element size for the
 * pair-per-thread kernel), heads per thread, and the CTA's (x, y, z) extent
 * (threads per head row, head groups, positions). `style` is an
 * ako_b200_rope_style. Follows the library's built-in choice (in the
 * measurement build, any override in force). Not part of the reference's
 * interface; it has no counterpart there.
 */
int ako_b200_rope_plan(int64_t batch, int64_t seq_len, int64_t n_heads, int64_t head_dim, int style, int dtype,
                       int* access_bytes, int* heads_per_thread, int* block_x, int* block_y, int* block_z);

/*
 * The launch a SwiGLU call of `n_rows` x `hidden_dim` in `dtype` would get,
 * without launching anything (host only; no GPU needed): bytes per access
 * (16; 4 for decode-sized problems; the element size when the operands are
 * not 16-byte aligned), threads per CTA, vectors per thread, and the grid's
 * budget of threads per SM (the grid strides over the problem with that many
 * threads for each SM; dense problems of 2^24 or more vectors keep at most
 * four CTAs on an SM at once and run the rest as those finish). `aligned`
 * says whether the call's pointers and row strides are 16-byte aligned,
 * `dense` whether all three operands are contiguous. Follows the library's
 * built-in choice (in the measurement build, any override in force). Not
 * part of the reference's interface; it has no counterpart there.
 */
int ako_b200_swiglu_plan(int64_t n_rows, int64_t hidden_dim, int dtype, int aligned, int dense,
                         int* access_bytes, int* threads, int* vectors_per_thread, int* threads_per_sm);

#ifdef __cplusplus
}
#endif

#endif /* AKO_B200_H_ */
