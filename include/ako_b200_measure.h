/*
 * ako_b200_measure.h — launch overrides of the measurement build.
 *
 * These functions are exported only by libako_b200_measure.so, a second build
 * of the same kernel sources compiled with AKO_B200_MEASUREMENT. It exports
 * every function of ako_b200.h as well, so a sweep, a benchmark or a test can
 * force a launch shape, a kernel or a launch mode and then call the ops of
 * the same library. The product library (libako_b200.so) compiles every
 * override as a constant at its built-in value; nothing a process does
 * through this header changes which kernel a call into the product library
 * runs, or its result.
 *
 * The overrides are process-wide plain settings of the measurement library:
 * set them from one thread while no call into it is in flight. None of them
 * is part of the reference's interface; they have no counterpart there.
 */
#ifndef AKO_B200_MEASURE_H_
#define AKO_B200_MEASURE_H_

#include "ako_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/*
 * RMSNorm launch shape: rows are split over `cluster` CTAs (1, 2, 4 or 8; a
 * thread-block cluster when > 1), each row slice held by `threads_per_row`
 * threads with `vectors_per_thread` 16-byte vectors each. (0, 0, 0) restores
 * the built-in table. A shape that cannot hold a given row, or that would
 * split it into slices of partial 32-vector groups, is ignored for that row.
 */
int ako_b200_rmsnorm_set_launch(int cluster, int threads_per_row, int vectors_per_thread);

/*
 * RMSNorm kernel choice: mode 1 uses the row-resident kernel only; mode 2
 * uses, where the row fits, the persistent kernel that stages rows in shared
 * memory with 1-D bulk copies (`stages` rows in flight per CTA, `ctas_per_sm`
 * CTAs per SM; 0 = defaults); mode 3 uses, for plain rows of 2049-8192
 * 16-byte vectors, the persistent kernel that streams each row through
 * shared memory in one or two chunks; mode 0 restores the built-in choice.
 */
int ako_b200_rmsnorm_set_staging(int mode, int stages, int ctas_per_sm);

/*
 * RMSNorm any-width kernel (rows that are not whole 16-byte vectors, or
 * pointers that are not 16-byte aligned): 32 threads per row (a warp per
 * row) or 256 (a CTA per row); 0 restores the built-in choice by row width.
 */
int ako_b200_rmsnorm_set_generic(int threads_per_row);

/*
 * Polls of the persistent kernels' bounded wait for a bulk copy (built-in:
 * 2^24, about a second). 0 makes every such wait run out at once, which
 * exercises the expiry path of ako_b200_take_device_status without any copy
 * failing: the copies still land and are drained before the kernel exits.
 * Returns the previous value.
 */
unsigned ako_b200_measure_set_wait_polls(unsigned polls);

/*
 * RoPE launch shape: each thread rotates `heads_per_thread` heads (1, 2 or
 * 4); 0 restores the built-in choice.
 */
int ako_b200_rope_set_launch(int heads_per_thread);

/*
 * SwiGLU launch shape: CTAs of `threads` threads (64, 128 or 256), each
 * keeping `vectors_per_thread` 16-byte vectors in flight (1, 2; 4 with 256
 * threads); (0, 0) restores the built-in choice.
 */
int ako_b200_swiglu_set_launch(int threads, int vectors_per_thread);

/*
 * SwiGLU grid budget: the grid-stride grid has at most `threads_per_sm`
 * threads for each SM (a multiple of 64 in [64, 8192]; above what an SM holds
 * at once, the CTAs run in several passes); 0 restores the built-in choice.
 */
int ako_b200_swiglu_set_grid(int threads_per_sm);

/*
 * SwiGLU CTAs request `bytes` of dynamic shared memory (in [0, 49152]), which
 * the kernel does not use: it caps how many CTAs an SM holds at once. 0
 * restores the built-in launch.
 */
int ako_b200_swiglu_set_smem(int bytes);

/*
 * Programmatic dependent launch: with `enable` = 1 (the built-in setting)
 * every kernel is launched with programmatic stream serialization, so it may
 * start while the previous kernel in the stream drains; it waits for that
 * kernel's completion before touching memory, so results do not change. 0
 * launches with plain stream order. Returns the previous setting.
 */
int ako_b200_set_pdl(int enable);

#ifdef __cplusplus
}
#endif

#endif /* AKO_B200_MEASURE_H_ */
