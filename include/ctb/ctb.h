/*
 * ctb.h — C ABI of the B200 (sm_100a) CUDA backend for ctorch's eager tensor-op hot path.
 *
 * These entry points are what ctorch's CUDA dispatch slots bind to. ctorch fills its CUDA slots
 * through four extern "C" registration hooks (src/ops/binary_ops_cpu.cpp:130,146,
 * src/ops/unary_ops_cpu.cpp:126,142, src/ops/reduction_ops_cpu.cpp:371,388,
 * src/ops/indexing_cpu.cpp:144,153); ctorch_b200/ctorch_plugin/cuda_backend.cpp defines those four
 * hooks and forwards each ctorch::Tensor to the functions below. No C++ or torch types cross this
 * boundary: every tensor is a ctb_view (device pointer + dtype + shape + element strides), every
 * failure is an int status, never an exception.
 *
 * Threading and streams: every call enqueues work on `stream` (NULL = the legacy default stream,
 * which is what ctorch's own CUDA kernels use) on the CURRENT device and returns without
 * synchronising, except where a function says otherwise. Calls are thread-safe; per-call state
 * lives in caller-provided scratch memory.
 *
 * Outputs are never allocated here: the caller passes them (ctorch's front-doors preallocate every
 * output, include/ctorch/ops/op_keys.h:30-32). Reductions may need scratch memory; the caller
 * sizes it with the matching *_scratch_bytes function (ctorch takes it from its CUDA caching
 * allocator, as its own CUDA backend does at src/ops/reduction_ops_cuda.cu:154-177).
 */
#ifndef CTB_CTB_H
#define CTB_CTB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CTB_MAX_DIMS 16 /* ctorch's kMaxRank (src/ops/tensor_iter.h:35) */

#if defined(_WIN32)
#define CTB_API __declspec(dllexport)
#else
#define CTB_API __attribute__((visibility("default")))
#endif
#define CTB_ABI_VERSION 1

/* Element types; the codes are the enumerator values of ctorch::dtype (include/ctorch/dtype.h:24-31). */
enum ctb_dtype { CTB_FLOAT32 = 0, CTB_FLOAT64 = 1, CTB_INT32 = 2, CTB_INT64 = 3, CTB_BOOL = 4,
                 CTB_BFLOAT16 = 5 };

/* Status codes. The ctorch shim maps them onto ctorch's exception tree (include/ctorch/errors.h). */
enum ctb_status {
    CTB_OK = 0,
    CTB_ERR_DTYPE = 1,    /* unsupported dtype combination          -> ctorch::DTypeError  */
    CTB_ERR_SHAPE = 2,    /* incompatible shapes / rank > 16 / axis -> ctorch::ShapeError  */
    CTB_ERR_INDEX = 3,    /* index_select index out of range        -> ctorch::ShapeError  */
    CTB_ERR_CUDA = 4,     /* CUDA runtime/launch error              -> ctorch::DeviceError */
    CTB_ERR_ARGUMENT = 5, /* null pointer, unknown op code          -> std::invalid_argument */
    CTB_ERR_SCRATCH = 6   /* scratch smaller than *_scratch_bytes reported */
};

/* Binary op codes (AddOp/SubOp/MulOp/DivOp, include/ctorch/ops/op_keys.h:35-46). */
enum ctb_binary_op { CTB_ADD = 0, CTB_SUB = 1, CTB_MUL = 2, CTB_DIV = 3 };
/* Unary op codes (NegOp..TanhOp, include/ctorch/ops/op_keys.h:69-92). */
enum ctb_unary_op { CTB_NEG = 0, CTB_ABS = 1, CTB_EXP = 2, CTB_LOG = 3, CTB_SQRT = 4,
                    CTB_RELU = 5, CTB_SIGMOID = 6, CTB_TANH = 7 };
/* Reduction op codes (SumOp/MeanOp/ProdOp/MaxValOp/MinValOp, op_keys.h:109-123). */
enum ctb_reduce_op { CTB_SUM = 0, CTB_MEAN = 1, CTB_PROD = 2, CTB_MAX = 3, CTB_MIN = 4 };

/* A strided tensor view on the current device. `data` is the address of element (0,...,0),
 * i.e. storage base + offset * itemsize (ctorch's offset is in elements, include/ctorch/tensor.h:33).
 * Strides are in elements and may be 0 (broadcast). ndim 0 is a scalar. */
typedef struct ctb_view {
    void* data;
    int32_t dtype;
    int32_t ndim;
    int64_t shape[CTB_MAX_DIMS];
    int64_t strides[CTB_MAX_DIMS];
} ctb_view;

/* Opaque cudaStream_t. */
typedef void* ctb_stream;

/* ABI version (CTB_ABI_VERSION of the built library). */
CTB_API int ctb_abi_version(void);

/* Message for the last non-OK status returned on the calling thread ("" if none). */
CTB_API const char* ctb_last_error(void);

/* Number of kernel launches this library has issued on the calling thread since the last
 * ctb_launch_count_reset(). Used by benchmarks to report how many of the library's kernels ran in
 * a timed region. */
CTB_API uint64_t ctb_launch_count(void);
CTB_API void ctb_launch_count_reset(void);

/* Number of waits that timed out on the current device since the library was loaded. Kernels that
 * stream through shared memory with bulk asynchronous copies (the column reductions of
 * ctb_reduce / ctb_reduce_index) bound every wait to about a second; a wait that runs out is
 * counted here, and the kernel returns without writing its outputs instead of hanging. A
 * healthy device reports 0. Synchronous (reads device memory). No ctorch counterpart: ctorch's
 * kernels have no waits. */
CTB_API int ctb_wait_timeouts(uint64_t* count);

/* out = op(a, b), elementwise with right-aligned broadcasting of a and b to out's shape.
 * Replaces ctorch's BinaryFn CUDA slots (include/ctorch/ops/op_keys.h:33-46; reference kernels
 * src/ops/binary_ops_cuda.cu:53-112) and, with out == a, the BinaryInplaceFn slots (:50-62).
 * a and b may be any strided views and may have different dtypes: each operand element is
 * converted to out's dtype in registers (static_cast semantics), and out's dtype must equal
 * promote_types(a, b) (src/type_promotion.cpp:45-62). Integer add/sub/mul wrap (two's
 * complement, src/ops/functors.h:39-66); integer div, bool and bfloat16 give CTB_ERR_DTYPE.
 * out may alias a or b only element-for-element (same data pointer and strides). */
CTB_API int ctb_binary(int op, const ctb_view* a, const ctb_view* b, const ctb_view* out,
               ctb_stream stream);

/* out = in converted to out's dtype, elementwise; out has in's shape and any strides. The
 * conversions of ctorch's cast (src/ops/cast_cpu.cpp:21-90): static_cast, bool read as 0/1, any
 * nonzero (NaN included) written to bool as true, float -> integer truncated toward zero. A NaN or
 * out-of-range float -> integer is undefined behaviour in ctorch (its x86 build gives the integer
 * minimum); here it saturates and NaN gives 0. With out's dtype equal to in's and out contiguous
 * this is a strided -> contiguous copy. It stands in for the host round trip of ctorch's CUDA
 * promotion (`maybe_cast`, src/ops/binary_ops_cpu.cpp:154-184, whose comment asks for a cast_cuda
 * kernel) and for the CPU-only strided materialisation of Tensor::contiguous()
 * (src/tensor.cpp:239-254). bfloat16 gives CTB_ERR_DTYPE. */
CTB_API int ctb_cast(const ctb_view* in, const ctb_view* out, ctb_stream stream);

/* out = op2(op1(a, b), c) in one pass, with the intermediate rounded to `mid_dtype` exactly as the
 * unfused pair of ctb_binary calls would round it (so results are bit-identical to the eager
 * sequence). mid_dtype must equal promote_types(a, b); out's dtype must equal
 * promote_types(mid_dtype, c). An eager-chain fusion with no single ctorch counterpart: it computes
 * ctorch's `op2(op1(a, b), c)` (two BinaryFn calls, src/ops/binary_ops_cpu.cpp:251-254) without
 * materialising the intermediate. */
CTB_API int ctb_binary_chain(int op1, int op2, const ctb_view* a, const ctb_view* b, const ctb_view* c,
                     int32_t mid_dtype, const ctb_view* out, ctb_stream stream);

/* out = unary_op(op(a, b)) in one pass (unary_op CTB_RELU, CTB_NEG or CTB_ABS), for a, b and out of
 * one dtype (int32/int64/float32/float64), broadcasting as ctb_binary. The binary result is rounded
 * to the dtype before the unary op sees it, so the result is bit-identical to ctorch's
 * relu(add(a, b)) and the like (two front-door calls, src/ops/binary_ops_cpu.cpp:251-254 and
 * src/ops/unary_ops_cpu.cpp:160-167) without writing and re-reading the intermediate. */
CTB_API int ctb_binary_unary(int op, int unary_op, const ctb_view* a, const ctb_view* b,
                             const ctb_view* out, ctb_stream stream);

/* out = op(in), same shape and dtype. Replaces the UnaryFn CUDA slots (op_keys.h:67-92; reference
 * src/ops/unary_ops_cuda.cu:50-101). neg/abs/relu accept int32/int64/float32/float64;
 * exp/log/sqrt/sigmoid/tanh accept float32/float64 only; bool and bfloat16 give CTB_ERR_DTYPE. */
CTB_API int ctb_unary(int op, const ctb_view* in, const ctb_view* out, ctb_stream stream);

/* Scratch bytes ctb_reduce needs for this problem (0 when none). */
CTB_API size_t ctb_reduce_scratch_bytes(int op, const ctb_view* in, const ctb_view* out,
                                uint32_t reduce_mask);

/* Multi-axis / whole-tensor reduction. Bit d of reduce_mask marks input dim d as reduced
 * (ctorch's ReductionAxes::reduce, src/ops/reduction.h:38-43). out has either the keepdim shape
 * (rank == in rank, 1 at reduced dims) or the kept dims only. Replaces the ReduceFn CUDA slots
 * (op_keys.h:99-123; reference src/ops/reduction_ops_cuda.cu:179-487). dtype rules
 * (src/ops/reduction.cpp:131-153): sum/prod of bool/int32/int64 -> int64, float passthrough with a
 * double accumulator for float32; mean is float-only; max/min keep the input dtype, propagate NaN
 * and return the first occurrence's bits on ties (so -0.0 vs +0.0 matches the sequential CPU
 * fold). Empty reductions write the identity (sum 0, prod 1, mean NaN, max -inf/lowest,
 * min +inf/highest), as ctorch's CPU kernel does. */
CTB_API int ctb_reduce(int op, const ctb_view* in, const ctb_view* out, uint32_t reduce_mask,
               void* scratch, size_t scratch_bytes, ctb_stream stream);

/* ctb_reduce without scratch from the caller, for callers that cannot allocate device memory:
 * a plain C or FFI host with no device allocator of its own to hand out scratch, or a process
 * that fixes its device memory at start-up and must not call cudaMalloc later (it can fail under
 * fragmentation and it synchronises the device). Same arguments, results and errors as
 * ctb_reduce; allocates nothing. Split reductions use a fixed 4 MiB array in the library's device
 * image instead (every GPU that loads the library holds it until exit); a reduction that would
 * need more returns CTB_ERR_SCRATCH and names the size. Each call that needs scratch looks up the
 * array's address on the current device (the first call on a device also loads the library's
 * device code there, so make that first call before any stream capture). All calls on a device share the one array and nothing in it needs
 * clearing between calls, but calls that overlap on the GPU (two streams, or two host threads)
 * race on it: serialise them. No counterpart in ctorch (ctorch's CUDA reductions always take
 * scratch from its caching allocator). */
CTB_API int ctb_reduce_noalloc(int op, const ctb_view* in, const ctb_view* out, uint32_t reduce_mask,
                               ctb_stream stream);

/* Scratch bytes ctb_reduce_index needs (0 when none). */
CTB_API size_t ctb_reduce_index_scratch_bytes(const ctb_view* in, int axis);

/* max/min along one axis with int64 indices (op = CTB_MAX / CTB_MIN). `values` may be NULL
 * (argmax/argmin). Replaces the ReduceWithIdxFn and ArgFn CUDA slots (op_keys.h:104-131;
 * reference src/ops/reduction_ops_cuda.cu:281-350). Semantics of
 * src/ops/reduction_ops_cpu.cpp:236-297: the first NaN wins, otherwise the first occurrence of
 * the extreme value. A zero-length axis gives CTB_ERR_SHAPE. */
CTB_API int ctb_reduce_index(int op, const ctb_view* in, const ctb_view* values, const ctb_view* indices,
                     int axis, void* scratch, size_t scratch_bytes, ctb_stream stream);

/* out = src gathered along `dim` by the 1-D int32/int64 `indices` (negative entries count from
 * the end). Replaces the IndexSelectFn CUDA slot (op_keys.h:139-148; reference
 * src/ops/indexing_cuda.cu:87-206). Every index is validated on the device before any row is
 * written; on a bad index nothing is written to out and *d_status (a device int32 the caller
 * owns) becomes nonzero. The call itself returns CTB_OK after enqueueing; the caller learns of a
 * bad index by reading *d_status once the stream has reached this point (ctorch's shim does that
 * synchronously and throws ShapeError, as ctorch's own CUDA path does at
 * src/ops/indexing_cuda.cu:186-194). d_status must point to 16 bytes of device memory: an int32
 * flag at byte 0 and, at byte 8, the int64 value of an offending index. */
CTB_API int ctb_index_select(const ctb_view* src, int dim, const ctb_view* indices, const ctb_view* out,
                     int32_t* d_status, ctb_stream stream);

/* ---- single-pass chain + row reductions ---- */

/* Scratch bytes for ctb_chain_rows (0 when d_sum is not wanted). */
CTB_API size_t ctb_chain_rows_scratch_bytes(int op1, int op2, const ctb_view* a, const ctb_view* b,
                                            const ctb_view* c, const ctb_view* y, int row_op,
                                            const ctb_view* row_index);

/* One pass over a [rows, cols] matrix a (unit inner stride) with b and c one broadcast row of
 * cols elements (or 0-d scalars), all float32 or all float64:
 *     y = op2(op1(a, b), c)                      written when y is not NULL
 *     row_index[r] = arg{min,max}_j y[r, j]      when row_index (int64 [rows]) is not NULL;
 *                                                row_op CTB_MIN or CTB_MAX
 *     *d_sum = sum of all y, in float64          when d_sum (device) is not NULL
 * Results equal ctorch's eager sequence on the same inputs: y = op2(op1(a, b), c) (two BinaryFn
 * calls, src/ops/binary_ops_cpu.cpp:251-254) bit for bit, row_index = argmin/argmax(y, -1)
 * (src/ops/reduction_ops_cpu.cpp:236-297: first index on ties, first NaN wins) bit for bit, and
 * the sum to float64 rounding (its own fixed order, so run-to-run identical). The eager sequence
 * reads y twice more; this reads a once and writes y once. */
CTB_API int ctb_chain_rows(int op1, int op2, const ctb_view* a, const ctb_view* b, const ctb_view* c,
                           const ctb_view* y, int row_op, const ctb_view* row_index, double* d_sum,
                           void* scratch, size_t scratch_bytes, ctb_stream stream);

/* ---- the one-pass step across GPUs: compute and the sum's exchange in one launch ---- */

/* Bytes of one rank's peer workspace (allocated by ctb_peer_alloc). */
CTB_API size_t ctb_peer_workspace_bytes(void);

/* Allocates this rank's peer workspace on the current device (zeroed) and writes its CUDA IPC
 * handle (64 bytes) to ipc_handle for the other ranks of the node. */
CTB_API int ctb_peer_alloc(void** d_workspace, void* ipc_handle);

/* Maps another rank's workspace (from its IPC handle) into this process. */
CTB_API int ctb_peer_open(const void* ipc_handle, void** d_peer_workspace);

/* Reads this rank's exchange status from its workspace (a synchronous device-to-host copy):
 * done_epoch = the last call whose exchange completed, failed_epoch = the last call whose wait
 * for another rank ran out (0: none). */
CTB_API int ctb_peer_status(const void* d_my_workspace, uint64_t* done_epoch, uint64_t* failed_epoch);

/* Copies this rank's per-call timestamps (a synchronous device-to-host copy) into out[64][4]:
 * row epoch % 64 holds, in ns of this GPU's %globaltimer, when CTA 0 of that call started, when
 * its first and its last CTA finished their rows, and when its exchange completed (or its wait
 * ran out). Rows of calls not yet made are 0. */
CTB_API int ctb_peer_trace(const void* d_my_workspace, uint64_t* out);

/* Unmaps a workspace opened with ctb_peer_open; frees this rank's own. */
CTB_API int ctb_peer_close(void* d_peer_workspace);
CTB_API int ctb_peer_free(void* d_workspace);

/* ctb_chain_rows over this rank's rows, with the whole-tensor sum taken across `world` ranks in
 * the same launch: the last CTA of the launch stores this rank's float64 partial over NVLink into
 * slot `rank` of every rank's workspace (d_peer_workspaces: device array of the world workspace
 * addresses, this rank's own at [rank]), waits until every rank's slot in its own workspace
 * carries `epoch`, and writes out_sum (0-d float32/float64) = the rank partials added in rank
 * order, the same on every rank, plus the partials to d_rank_partials [world] when not NULL.
 * Every rank makes the same calls with epoch = 1, 2, 3, ..., each rank's calls in stream order.
 * The slots are double-buffered by epoch parity and a slot is taken only when it carries exactly
 * `epoch`, so a rank that runs one call ahead never feeds a slower rank its next partial. Each
 * wait is bounded by timeout_ns (0: one second); a wait that runs out is counted
 * (ctb_wait_timeouts), recorded in the workspace (ctb_peer_status: failed_epoch) and leaves NaN
 * in out_sum and in the missing ranks' d_rank_partials. The ranks must run on different GPUs. No ctorch counterpart (ctorch has no
 * multi-GPU layer); per rank it is ctb_chain_rows, and the sum is ctorch's whole-tensor sum
 * (src/ops/reduction_ops_cpu.cpp:463) of the row-sharded y. */
CTB_API int ctb_chain_rows_allsum(int op1, int op2, const ctb_view* a, const ctb_view* b, const ctb_view* c,
                                  const ctb_view* y, int row_op, const ctb_view* row_index,
                                  void* const* d_peer_workspaces, void* d_my_workspace, int rank, int world,
                                  uint64_t epoch, const ctb_view* out_sum, double* d_rank_partials,
                                  uint64_t timeout_ns, ctb_stream stream);

/* ---- sharded reductions (multi-GPU layer) ---- */

/* Scratch bytes for ctb_sum_partial. */
CTB_API size_t ctb_sum_partial_scratch_bytes(const ctb_view* in);

/* Whole-tensor sum of a float32/float64 shard into one float64 partial at d_partial (device).
 * Per-shard step of a row-sharded `sum` (ctorch's whole-tensor sum,
 * src/ops/reduction_ops_cpu.cpp:463) whose partials are combined across GPUs. */
CTB_API int ctb_sum_partial(const ctb_view* in, double* d_partial, void* scratch, size_t scratch_bytes,
                    ctb_stream stream);

/* out (0-d, float32 or float64) = the sum of n float64 partials taken in index order, rounded
 * once to out's dtype. Deterministic for a fixed n. */
CTB_API int ctb_sum_combine(const double* d_partials, int n, const ctb_view* out, ctb_stream stream);

/* Combine step of a row-sharded max/min over dim 0 (op = CTB_MAX / CTB_MIN): values [G, N] and
 * int64 indices [G, N] hold the G shards' own results (row g = rank g's ctb_reduce_index output,
 * indices local to its shard); d_row_offsets is a device int64 array of the G shards' first global
 * rows. Writes out_indices [N] (global rows) and, unless NULL, out_values [N], combining the shards
 * in rank order with ctorch's rule: the first NaN wins, otherwise the first occurrence of the
 * extreme value (src/ops/reduction_ops_cpu.cpp:236-297). The result equals the single-GPU
 * reduction of the whole tensor. No ctorch counterpart (ctorch has no multi-GPU layer). */
CTB_API int ctb_minmax_combine(int op, const ctb_view* values, const ctb_view* indices,
                               const int64_t* d_row_offsets, const ctb_view* out_values,
                               const ctb_view* out_indices, ctb_stream stream);

/* ---- synthetic inputs ---- */

/* Fills a contiguous view with a counter-based pseudo-random sequence (splitmix64 of
 * (seed, stream_id, element index)); the same element gets the same value however the tensor is
 * sharded if `first_index` is its global position. dist 0 = uniform [lo, hi) (float) or integer
 * uniform [lo, hi] (int), dist 1 = normal(lo, hi) by Box-Muller (float only). */
CTB_API int ctb_fill_random(const ctb_view* out, int dist, uint64_t seed, uint64_t stream_id,
                    int64_t first_index, double lo, double hi, ctb_stream stream);

#ifdef __cplusplus
}
#endif

#endif /* CTB_CTB_H */
