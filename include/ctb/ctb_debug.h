/*
 * ctb_debug.h — host-only introspection of the B200 backend's planner, plus a GPU self-test of
 * the bounded wait. The planner functions make no CUDA call that needs a device, so the planner
 * can be tested on a machine without a GPU. They have no counterpart in ctorch (ctorch builds its iteration plans inline:
 * src/ops/tensor_iter.cpp:41-84, src/ops/reduction_iter.cpp:20-69).
 */
#ifndef CTB_CTB_DEBUG_H
#define CTB_CTB_DEBUG_H

#include "ctb/ctb.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Plans out = f(ins...) as ctb_binary / ctb_unary / ctb_binary_chain would and reports the launch
 * shape ("empty", "flat", "rows_long", "rows_short", "tiled", "general"), the collapsed rank and
 * the collapsed shape (shape must hold 16 entries). `vec` is the pack width in elements. */
CTB_API int ctb_debug_plan_elementwise(const ctb_view* out, const ctb_view* const* ins, int nin, int vec,
                               char* path, int path_len, int* rank, int64_t* shape);

/* Plans a reduction and reports "empty", "inner", "outer" or "general" and the collapsed ranks. */
CTB_API int ctb_debug_plan_reduction(const ctb_view* in, const ctb_view* out, uint32_t reduce_mask,
                             char* path, int path_len, int* rank_kept, int* rank_red);

/* The strip column kernel's geometry rule, without a device: for `batch` rows of `np` 16-byte
 * packs over `slots` CTAs, with strips at most `pk_max` packs wide, 1 and the strip count and
 * widest strip when the kernel takes the shape, else 0. */
CTB_API int ctb_debug_strip_geometry(int64_t batch, int64_t np, int64_t pk_max, int64_t slots,
                                     int64_t* strips, int64_t* pk);

/* Copies into `buf` the name of the first kernel that the calling thread's last reduction
 * launched ("red_cols_strip", "red_cols_bulk", "red_inner_warp", ...; "" before any). */
CTB_API int ctb_debug_last_reduction_kernel(char* buf, int len);

/* floor(n / d) through the kernels' invariant-divisor multiply (n < 2^63, d >= 1). */
CTB_API uint64_t ctb_debug_fastdiv(uint64_t n, uint64_t d);

/* The size check of ctb_reduce_noalloc, without a device: CTB_OK when a reduction needing `need`
 * bytes of scratch fits its fixed 4 MiB array, else CTB_ERR_SCRATCH with the message the entry
 * point gives (ctb_last_error). */
CTB_API int ctb_debug_noalloc_fits(size_t need);

/* Self-test of the bounded wait (needs a GPU, unlike the functions above): one thread waits on a
 * shared-memory barrier that nothing arrives at, for limit_ns (at most 100 ms), then returns.
 * *completed is 0 when the wait timed out, as it must; the timeout is also counted by
 * ctb_wait_timeouts. Synchronous. */
CTB_API int ctb_debug_wait_timeout(uint64_t limit_ns, int* completed);

#ifdef __cplusplus
}
#endif

#endif /* CTB_CTB_DEBUG_H */
