// capi.cu — the extern "C" entry points of include/ctb/ctb.h: argument and dtype validation
// (mirroring the checks ctorch's CUDA backend makes before launching), then dispatch to the
// kernel families. No exception ever leaves this file.
#include <atomic>
#include <cstdio>
#include <exception>
#include <map>
#include <mutex>
#include <string>
#include <tuple>

#include "common.cuh"
#include "peer.cuh"
#include "plan.cuh"

namespace ctb {

template <int OP> int binary_dispatch(const ctb_view*, const ctb_view*, const ctb_view*, cudaStream_t);
int fused_chain_rows(int op1, int op2, const ctb_view* a, const ctb_view* b, const ctb_view* c,
                     const ctb_view* out, cudaStream_t st);  // fused_rows.cu; -1 when it does not apply
extern template int binary_dispatch<CTB_ADD>(const ctb_view*, const ctb_view*, const ctb_view*, cudaStream_t);
extern template int binary_dispatch<CTB_SUB>(const ctb_view*, const ctb_view*, const ctb_view*, cudaStream_t);
extern template int binary_dispatch<CTB_MUL>(const ctb_view*, const ctb_view*, const ctb_view*, cudaStream_t);
extern template int binary_dispatch<CTB_DIV>(const ctb_view*, const ctb_view*, const ctb_view*, cudaStream_t);
int unary_dispatch(int op, const ctb_view* in, const ctb_view* out, cudaStream_t st);
int bin_unary_dispatch(int op, int uop, const ctb_view* a, const ctb_view* b, const ctb_view* out,
                       cudaStream_t st);
int chain_dispatch(int op1, int op2, const ctb_view* a, const ctb_view* b, const ctb_view* c,
                   const ctb_view* out, cudaStream_t st);
int sum_like_dispatch(int op, const ctb_view* in, const ctb_view* out, uint32_t mask, void* scratch,
                      size_t sb, cudaStream_t st, size_t* need_only);
int minmax_dispatch(int op, const ctb_view* in, const ctb_view* values, const ctb_view* indices,
                    uint32_t mask, void* scratch, size_t sb, cudaStream_t st, size_t* need_only);
int sum_partial_dispatch(const ctb_view* in, double* d_partial, void* scratch, size_t sb,
                         cudaStream_t st, size_t* need_only);
int sum_combine(const double* parts, int n, const ctb_view* out, cudaStream_t st);
int fused_rows_allsum(int op1, int op2, const ctb_view* a, const ctb_view* b, const ctb_view* c,
                      const ctb_view* y, int row_op, const ctb_view* idx, PeerWorkspace* const* d_peers,
                      int rank, int world, uint64_t epoch, const ctb_view* out_sum, double* d_parts,
                      uint64_t timeout_ns, unsigned long long* timeouts, PeerWorkspace* my_ws, cudaStream_t st);
unsigned long long* wait_timeout_counter();
int cast_dispatch(const ctb_view* in, const ctb_view* out, cudaStream_t st);
int minmax_combine(int op, const ctb_view* values, const ctb_view* indices, const int64_t* d_offsets,
                   const ctb_view* out_values, const ctb_view* out_indices, cudaStream_t st);
int index_select_dispatch(const ctb_view* src, int dim, const ctb_view* idx, const ctb_view* out,
                          int32_t* status, cudaStream_t st);
int fill_random(const ctb_view* out, int dist, uint64_t seed, uint64_t stream_id, int64_t first,
                double lo, double hi, cudaStream_t st);
int reduce_noalloc(int op, const ctb_view* in, const ctb_view* out, uint32_t mask, cudaStream_t st);
size_t fused_rows_scratch(int op1, int op2, const ctb_view* a, const ctb_view* b, const ctb_view* c,
                          const ctb_view* y, int row_op, const ctb_view* idx);
int fused_rows(int op1, int op2, const ctb_view* a, const ctb_view* b, const ctb_view* c,
               const ctb_view* y, int row_op, const ctb_view* idx, double* d_sum, void* scratch,
               size_t scratch_bytes, cudaStream_t st);

namespace {
thread_local std::string t_error;
thread_local uint64_t t_launches = 0;
}  // namespace

int fail(int status, const std::string& msg) {
    t_error = msg;
    return status;
}

int check_launch(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return fail(CTB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
    return CTB_OK;
}

void count_launch(int n) { t_launches += static_cast<uint64_t>(n); }

int sm_count() {
    static std::mutex mu;
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    std::lock_guard<std::mutex> lock(mu);
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

int resident_ctas(const void* fn, int block, size_t smem) {
    static std::mutex mu;
    static std::map<std::tuple<const void*, int, int, size_t>, int> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return 4;
    }
    const auto key = std::make_tuple(fn, dev, block, smem);
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, block, smem) != cudaSuccess || n < 1) {
        cudaGetLastError();
        n = 1;
    }
    cache[key] = n;
    return n;
}

size_t dtype_size(int dt) {
    switch (dt) {
    case CTB_FLOAT32: return 4;
    case CTB_FLOAT64: return 8;
    case CTB_INT32: return 4;
    case CTB_INT64: return 8;
    case CTB_BOOL: return 1;
    case CTB_BFLOAT16: return 2;
    }
    return 0;
}

const char* dtype_name(int dt) {
    switch (dt) {
    case CTB_FLOAT32: return "float32";
    case CTB_FLOAT64: return "float64";
    case CTB_INT32: return "int32";
    case CTB_INT64: return "int64";
    case CTB_BOOL: return "bool";
    case CTB_BFLOAT16: return "bfloat16";
    }
    return "unknown";
}

// src/type_promotion.cpp:45-62
int promote(int a, int b) {
    static const int rank_of[5] = {3, 4, 1, 2, 0};  // f32, f64, i32, i64, bool
    static const int dtype_of_rank[5] = {CTB_BOOL, CTB_INT32, CTB_INT64, CTB_FLOAT32, CTB_FLOAT64};
    if (a < 0 || a > 4 || b < 0 || b > 4) return -1;
    const int ra = rank_of[a], rb = rank_of[b];
    return dtype_of_rank[ra > rb ? ra : rb];
}

static bool valid_view(const ctb_view* v) {
    if (!v) return false;
    if (v->ndim < 0 || v->ndim > kMaxDims) return false;
    for (int d = 0; d < v->ndim; ++d)
        if (v->shape[d] < 0) return false;
    return v->dtype >= 0 && v->dtype <= CTB_BFLOAT16;
}

static int64_t view_numel(const ctb_view* v) {
    int64_t n = 1;
    for (int d = 0; d < v->ndim; ++d) n *= v->shape[d];
    return n;
}

static int check_views(std::initializer_list<const ctb_view*> vs) {
    for (const ctb_view* v : vs) {
        if (!v) return fail(CTB_ERR_ARGUMENT, "null view");
        if (v->ndim < 0 || v->ndim > kMaxDims)
            return fail(CTB_ERR_SHAPE, "CUDA backend does not support tensor rank > 16 (got " +
                                           std::to_string(v->ndim) + ")");
        if (!valid_view(v)) return fail(CTB_ERR_ARGUMENT, "malformed view");
        if (v->data == nullptr && view_numel(v) != 0) return fail(CTB_ERR_ARGUMENT, "null data pointer");
    }
    return CTB_OK;
}

template <class F> static int guarded(F&& f) {
    try {
        return f();
    } catch (const std::exception& e) {
        return fail(CTB_ERR_CUDA, std::string("internal error: ") + e.what());
    } catch (...) {
        return fail(CTB_ERR_CUDA, "internal error");
    }
}

}  // namespace ctb

using namespace ctb;

extern "C" {

int ctb_abi_version(void) { return CTB_ABI_VERSION; }

const char* ctb_last_error(void) { return t_error.c_str(); }

uint64_t ctb_launch_count(void) { return t_launches; }
void ctb_launch_count_reset(void) { t_launches = 0; }

int ctb_binary(int op, const ctb_view* a, const ctb_view* b, const ctb_view* out, ctb_stream stream) {
    return guarded([&]() -> int {
        t_error.clear();
        if (int rc = check_views({a, b, out})) return rc;
        if (op < CTB_ADD || op > CTB_DIV) return fail(CTB_ERR_ARGUMENT, "unknown binary op");
        // src/ops/binary_ops_cuda.cu:115-154 / binary_ops_cpu.cpp:81-85,106-109,202-208
        if (a->dtype == CTB_BOOL || b->dtype == CTB_BOOL || out->dtype == CTB_BOOL)
            return fail(CTB_ERR_DTYPE, "binary arithmetic on bool is not supported (promote to int32 first)");
        if (a->dtype == CTB_BFLOAT16 || b->dtype == CTB_BFLOAT16 || out->dtype == CTB_BFLOAT16)
            return fail(CTB_ERR_DTYPE, "bfloat16 is not supported");
        const int pt = promote(a->dtype, b->dtype);
        if (pt != out->dtype)
            return fail(CTB_ERR_DTYPE, std::string("output dtype ") + dtype_name(out->dtype) +
                                           " is not the promoted dtype " + dtype_name(pt));
        if (op == CTB_DIV && (out->dtype == CTB_INT32 || out->dtype == CTB_INT64))
            return fail(CTB_ERR_DTYPE, "integer division is not supported; cast operands to float32/float64 first");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        // A float matrix of at least 16384 contiguous rows of 32 KiB or more and b one broadcast row
        // of the same dtype: the row kernel of the chain, software-pipelined at the copy rate
        // (config 5's X - r: 2585 us against 2720-2746 us for the elementwise row tiles).
        if ((out->dtype == CTB_FLOAT32 || out->dtype == CTB_FLOAT64) && a->dtype == out->dtype &&
            b->dtype == out->dtype && out->ndim >= 1 && out->shape[out->ndim - 1] > 1) {
            int64_t nb = 1;
            for (int d = 0; d < b->ndim; ++d) nb *= b->shape[d];
            if (nb == out->shape[out->ndim - 1]) {
                const int rc = fused_chain_rows(op, kOpNone, a, b, b, out, st);
                if (rc != -1) return rc;
            }
        }
        switch (op) {
        case CTB_ADD: return binary_dispatch<CTB_ADD>(a, b, out, st);
        case CTB_SUB: return binary_dispatch<CTB_SUB>(a, b, out, st);
        case CTB_MUL: return binary_dispatch<CTB_MUL>(a, b, out, st);
        default: return binary_dispatch<CTB_DIV>(a, b, out, st);
        }
    });
}

int ctb_binary_chain(int op1, int op2, const ctb_view* a, const ctb_view* b, const ctb_view* c,
                     int32_t mid_dtype, const ctb_view* out, ctb_stream stream) {
    return guarded([&]() -> int {
        t_error.clear();
        if (int rc = check_views({a, b, c, out})) return rc;
        if (op1 < CTB_ADD || op1 > CTB_DIV || op2 < CTB_ADD || op2 > CTB_DIV)
            return fail(CTB_ERR_ARGUMENT, "unknown binary op");
        const int dt = out->dtype;
        if ((dt != CTB_FLOAT32 && dt != CTB_FLOAT64) || a->dtype != dt || b->dtype != dt ||
            c->dtype != dt || mid_dtype != dt)
            return fail(CTB_ERR_DTYPE, "fused chains take float32 or float64 operands of one dtype");
        return chain_dispatch(op1, op2, a, b, c, out, static_cast<cudaStream_t>(stream));
    });
}

int ctb_binary_unary(int op, int unary_op, const ctb_view* a, const ctb_view* b, const ctb_view* out,
                     ctb_stream stream) {
    return guarded([&]() -> int {
        t_error.clear();
        if (int rc = check_views({a, b, out})) return rc;
        if (op < CTB_ADD || op > CTB_DIV) return fail(CTB_ERR_ARGUMENT, "unknown binary op");
        if (unary_op != CTB_RELU && unary_op != CTB_NEG && unary_op != CTB_ABS)
            return fail(CTB_ERR_ARGUMENT, "the fused unary op must be relu, neg or abs");
        const int dt = out->dtype;
        if (a->dtype != dt || b->dtype != dt ||
            (dt != CTB_FLOAT32 && dt != CTB_FLOAT64 && dt != CTB_INT32 && dt != CTB_INT64))
            return fail(CTB_ERR_DTYPE, "binary+unary chains take int32/int64/float32/float64 operands of one dtype");
        if (op == CTB_DIV && (dt == CTB_INT32 || dt == CTB_INT64))
            return fail(CTB_ERR_DTYPE, "integer division is not supported; cast operands to float32/float64 first");
        return bin_unary_dispatch(op, unary_op, a, b, out, static_cast<cudaStream_t>(stream));
    });
}

int ctb_unary(int op, const ctb_view* in, const ctb_view* out, ctb_stream stream) {
    return guarded([&]() -> int {
        t_error.clear();
        if (int rc = check_views({in, out})) return rc;
        if (op < CTB_NEG || op > CTB_TANH) return fail(CTB_ERR_ARGUMENT, "unknown unary op");
        if (in->dtype != out->dtype) return fail(CTB_ERR_DTYPE, "unary output dtype must equal the input dtype");
        if (in->ndim != out->ndim) return fail(CTB_ERR_SHAPE, "unary output shape must equal the input shape");
        for (int d = 0; d < in->ndim; ++d)
            if (in->shape[d] != out->shape[d]) return fail(CTB_ERR_SHAPE, "unary output shape must equal the input shape");
        const int dt = in->dtype;
        // src/ops/unary_ops_cuda.cu:103-143
        if (dt == CTB_BOOL) return fail(CTB_ERR_DTYPE, "not defined on bool — promote to int32 first");
        if (dt == CTB_BFLOAT16) return fail(CTB_ERR_DTYPE, "bfloat16 is not supported");
        const bool int_ok = op == CTB_NEG || op == CTB_ABS || op == CTB_RELU;
        if (!int_ok && (dt == CTB_INT32 || dt == CTB_INT64))
            return fail(CTB_ERR_DTYPE, "only float32/float64 inputs are supported");
        return unary_dispatch(op, in, out, static_cast<cudaStream_t>(stream));
    });
}

int ctb_cast(const ctb_view* in, const ctb_view* out, ctb_stream stream) {
    return guarded([&]() -> int {
        t_error.clear();
        if (int rc = check_views({in, out})) return rc;
        // src/ops/cast_cpu.cpp:62-90
        if (in->dtype == CTB_BFLOAT16) return fail(CTB_ERR_DTYPE, "ctorch: cast from bfloat16 not supported");
        if (out->dtype == CTB_BFLOAT16) return fail(CTB_ERR_DTYPE, "ctorch: cast to bfloat16 not supported");
        if (in->ndim != out->ndim) return fail(CTB_ERR_SHAPE, "cast output shape must equal the input shape");
        for (int d = 0; d < in->ndim; ++d)
            if (in->shape[d] != out->shape[d]) return fail(CTB_ERR_SHAPE, "cast output shape must equal the input shape");
        return cast_dispatch(in, out, static_cast<cudaStream_t>(stream));
    });
}

static int reduce_checks(int op, const ctb_view* in, const ctb_view* out) {
    if (int rc = check_views({in, out})) return rc;
    if (op < CTB_SUM || op > CTB_MIN) return fail(CTB_ERR_ARGUMENT, "unknown reduction op");
    const int dt = in->dtype;
    if (dt == CTB_BFLOAT16) return fail(CTB_ERR_DTYPE, "bfloat16 reductions are not supported");
    const bool is_float = dt == CTB_FLOAT32 || dt == CTB_FLOAT64;
    int want = dt;
    if (op == CTB_SUM || op == CTB_PROD) want = is_float ? dt : CTB_INT64;
    if (op == CTB_MEAN && !is_float) return fail(CTB_ERR_DTYPE, "mean requires a floating dtype input");
    if (out->dtype != want)
        return fail(CTB_ERR_DTYPE, std::string("reduction output dtype must be ") + dtype_name(want));
    return CTB_OK;
}

size_t ctb_reduce_scratch_bytes(int op, const ctb_view* in, const ctb_view* out, uint32_t mask) {
    size_t need = 0;
    const int rc = guarded([&]() -> int {
        if (int r = reduce_checks(op, in, out)) return r;
        if (op == CTB_MAX || op == CTB_MIN)
            return minmax_dispatch(op, in, out, nullptr, mask, nullptr, 0, nullptr, &need);
        return sum_like_dispatch(op, in, out, mask, nullptr, 0, nullptr, &need);
    });
    return rc == CTB_OK ? need : 0;
}

int ctb_reduce(int op, const ctb_view* in, const ctb_view* out, uint32_t mask, void* scratch,
               size_t scratch_bytes, ctb_stream stream) {
    return guarded([&]() -> int {
        t_error.clear();
        if (int r = reduce_checks(op, in, out)) return r;
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        if (op == CTB_MAX || op == CTB_MIN)
            return minmax_dispatch(op, in, out, nullptr, mask, scratch, scratch_bytes, st, nullptr);
        return sum_like_dispatch(op, in, out, mask, scratch, scratch_bytes, st, nullptr);
    });
}

int ctb_reduce_noalloc(int op, const ctb_view* in, const ctb_view* out, uint32_t mask,
                       ctb_stream stream) {
    return guarded([&]() -> int {
        t_error.clear();
        if (int r = reduce_checks(op, in, out)) return r;
        return reduce_noalloc(op, in, out, mask, static_cast<cudaStream_t>(stream));
    });
}

static int reduce_index_checks(int op, const ctb_view* in, const ctb_view* values,
                               const ctb_view* indices, int axis) {
    if (int rc = check_views({in, indices})) return rc;
    if (values)
        if (int rc = check_views({values})) return rc;
    if (op != CTB_MAX && op != CTB_MIN) return fail(CTB_ERR_ARGUMENT, "op must be CTB_MAX or CTB_MIN");
    if (in->dtype == CTB_BFLOAT16) return fail(CTB_ERR_DTYPE, "bfloat16 reductions are not supported");
    if (indices->dtype != CTB_INT64) return fail(CTB_ERR_DTYPE, "indices must be int64");
    if (values && values->dtype != in->dtype) return fail(CTB_ERR_DTYPE, "values dtype must equal the input dtype");
    if (in->ndim == 0) return fail(CTB_ERR_SHAPE, "cannot reduce a 0-d tensor along a single axis");
    if (axis < 0 || axis >= in->ndim) return fail(CTB_ERR_SHAPE, "axis out of range");
    if (in->shape[axis] == 0)
        return fail(CTB_ERR_SHAPE, "cannot reduce a zero-length axis (operation has no identity)");
    return CTB_OK;
}

size_t ctb_reduce_index_scratch_bytes(const ctb_view* in, int axis) {
    size_t need = 0;
    guarded([&]() -> int {
        if (!in || in->ndim <= 0 || in->ndim > kMaxDims || axis < 0 || axis >= in->ndim) return CTB_ERR_SHAPE;
        // plan with a keepdim-shaped index view (strides only matter for the plan's shape checks)
        ctb_view idx{};
        idx.dtype = CTB_INT64;
        idx.ndim = in->ndim;
        int64_t expect = 1;
        for (int d = in->ndim - 1; d >= 0; --d) {
            idx.shape[d] = d == axis ? 1 : in->shape[d];
            idx.strides[d] = expect;
            expect *= idx.shape[d];
        }
        return minmax_dispatch(CTB_MAX, in, nullptr, &idx, 1u << axis, nullptr, 0, nullptr, &need);
    });
    return need;
}

int ctb_reduce_index(int op, const ctb_view* in, const ctb_view* values, const ctb_view* indices,
                     int axis, void* scratch, size_t scratch_bytes, ctb_stream stream) {
    return guarded([&]() -> int {
        t_error.clear();
        if (int r = reduce_index_checks(op, in, values, indices, axis)) return r;
        return minmax_dispatch(op, in, values, indices, 1u << axis, scratch, scratch_bytes,
                               static_cast<cudaStream_t>(stream), nullptr);
    });
}

int ctb_index_select(const ctb_view* src, int dim, const ctb_view* indices, const ctb_view* out,
                     int32_t* d_status, ctb_stream stream) {
    return guarded([&]() -> int {
        t_error.clear();
        if (int rc = check_views({src, indices, out})) return rc;
        if (!d_status) return fail(CTB_ERR_ARGUMENT, "null status pointer");
        // src/ops/indexing_cpu.cpp:163-200, src/ops/indexing_cuda.cu:137-145
        if (indices->ndim != 1)
            return fail(CTB_ERR_SHAPE, "indices must be 1-D (got rank " + std::to_string(indices->ndim) + ")");
        if (indices->dtype != CTB_INT32 && indices->dtype != CTB_INT64)
            return fail(CTB_ERR_DTYPE, "indices dtype must be int32 or int64");
        if (src->dtype == CTB_BFLOAT16) return fail(CTB_ERR_DTYPE, "bfloat16 is not supported");
        if (out->dtype != src->dtype) return fail(CTB_ERR_DTYPE, "output dtype must equal the source dtype");
        if (src->ndim == 0) return fail(CTB_ERR_SHAPE, "cannot index a 0-d tensor");
        if (dim < 0 || dim >= src->ndim)
            return fail(CTB_ERR_SHAPE, "dim " + std::to_string(dim) + " out of range for tensor of rank " +
                                           std::to_string(src->ndim));
        if (out->ndim != src->ndim) return fail(CTB_ERR_SHAPE, "output rank must equal the source rank");
        for (int d = 0; d < src->ndim; ++d) {
            const int64_t want = d == dim ? indices->shape[0] : src->shape[d];
            if (out->shape[d] != want) return fail(CTB_ERR_SHAPE, "output shape mismatch");
        }
        return index_select_dispatch(src, dim, indices, out, d_status, static_cast<cudaStream_t>(stream));
    });
}

size_t ctb_chain_rows_scratch_bytes(int op1, int op2, const ctb_view* a, const ctb_view* b,
                                    const ctb_view* c, const ctb_view* y, int row_op,
                                    const ctb_view* row_index) {
    size_t need = 0;
    guarded([&]() -> int {
        if (check_views({a, b, c})) return CTB_ERR_ARGUMENT;
        need = fused_rows_scratch(op1, op2, a, b, c, y, row_op, row_index);
        return CTB_OK;
    });
    return need;
}

int ctb_chain_rows(int op1, int op2, const ctb_view* a, const ctb_view* b, const ctb_view* c,
                   const ctb_view* y, int row_op, const ctb_view* row_index, double* d_sum,
                   void* scratch, size_t scratch_bytes, ctb_stream stream) {
    return guarded([&]() -> int {
        t_error.clear();
        if (int rc = check_views({a, b, c})) return rc;
        if (y)
            if (int rc = check_views({y})) return rc;
        if (row_index)
            if (int rc = check_views({row_index})) return rc;
        return fused_rows(op1, op2, a, b, c, y, row_op, row_index, d_sum, scratch, scratch_bytes,
                          static_cast<cudaStream_t>(stream));
    });
}

size_t ctb_sum_partial_scratch_bytes(const ctb_view* in) {
    size_t need = 0;
    guarded([&]() -> int {
        if (!in || (in->dtype != CTB_FLOAT32 && in->dtype != CTB_FLOAT64)) return CTB_ERR_DTYPE;
        double dummy;
        return sum_partial_dispatch(in, &dummy, nullptr, 0, nullptr, &need);
    });
    return need;
}

int ctb_chain_rows_allsum(int op1, int op2, const ctb_view* a, const ctb_view* b, const ctb_view* c,
                          const ctb_view* y, int row_op, const ctb_view* row_index, void* const* d_peer_workspaces,
                          void* d_my_workspace, int rank, int world, uint64_t epoch, const ctb_view* out_sum,
                          double* d_rank_partials, uint64_t timeout_ns, ctb_stream stream) {
    return guarded([&]() -> int {
        t_error.clear();
        if (int rc = check_views({a, b, c, out_sum})) return rc;
        if (y)
            if (int rc = check_views({y})) return rc;
        if (row_index)
            if (int rc = check_views({row_index})) return rc;
        if (!d_peer_workspaces || !d_my_workspace) return fail(CTB_ERR_ARGUMENT, "null workspace");
        if (world < 1 || world > kPeerMaxRanks || rank < 0 || rank >= world)
            return fail(CTB_ERR_ARGUMENT, "rank/world out of range (world <= " + std::to_string(kPeerMaxRanks) + ")");
        if (epoch == 0) return fail(CTB_ERR_ARGUMENT, "epoch must start at 1 and grow by one per call");
        if (out_sum->dtype != CTB_FLOAT32 && out_sum->dtype != CTB_FLOAT64)
            return fail(CTB_ERR_DTYPE, "the sum must be float32 or float64");
        if (view_numel(out_sum) != 1) return fail(CTB_ERR_SHAPE, "the sum output must hold one element");
        unsigned long long* counter = wait_timeout_counter();
        if (!counter) return fail(CTB_ERR_CUDA, "device timeout counter unavailable");
        return fused_rows_allsum(op1, op2, a, b, c, y, row_op, row_index,
                                 reinterpret_cast<PeerWorkspace* const*>(d_peer_workspaces), rank, world, epoch,
                                 out_sum, d_rank_partials, timeout_ns ? timeout_ns : 1000000000ull, counter,
                                 static_cast<PeerWorkspace*>(d_my_workspace), static_cast<cudaStream_t>(stream));
    });
}

int ctb_sum_partial(const ctb_view* in, double* d_partial, void* scratch, size_t scratch_bytes,
                    ctb_stream stream) {
    return guarded([&]() -> int {
        t_error.clear();
        if (int rc = check_views({in})) return rc;
        if (!d_partial) return fail(CTB_ERR_ARGUMENT, "null partial pointer");
        if (in->dtype != CTB_FLOAT32 && in->dtype != CTB_FLOAT64)
            return fail(CTB_ERR_DTYPE, "partial sums take float32/float64 input");
        return sum_partial_dispatch(in, d_partial, scratch, scratch_bytes,
                                    static_cast<cudaStream_t>(stream), nullptr);
    });
}

int ctb_sum_combine(const double* d_partials, int n, const ctb_view* out, ctb_stream stream) {
    return guarded([&]() -> int {
        t_error.clear();
        if (int rc = check_views({out})) return rc;
        if (!d_partials || n < 0) return fail(CTB_ERR_ARGUMENT, "bad partials");
        if (out->dtype != CTB_FLOAT32 && out->dtype != CTB_FLOAT64)
            return fail(CTB_ERR_DTYPE, "combined sum must be float32/float64");
        if (view_numel(out) != 1) return fail(CTB_ERR_SHAPE, "combined sum output must hold one element");
        return sum_combine(d_partials, n, out, static_cast<cudaStream_t>(stream));
    });
}

int ctb_minmax_combine(int op, const ctb_view* values, const ctb_view* indices, const int64_t* d_row_offsets,
                       const ctb_view* out_values, const ctb_view* out_indices, ctb_stream stream) {
    return guarded([&]() -> int {
        t_error.clear();
        if (op != CTB_MAX && op != CTB_MIN) return fail(CTB_ERR_ARGUMENT, "op must be CTB_MAX or CTB_MIN");
        if (int rc = check_views({values, indices, out_indices})) return rc;
        if (out_values)
            if (int rc = check_views({out_values})) return rc;
        if (!d_row_offsets) return fail(CTB_ERR_ARGUMENT, "null row offsets");
        if (values->ndim != 2 || indices->ndim != 2 || out_indices->ndim != 1 || (out_values && out_values->ndim != 1))
            return fail(CTB_ERR_SHAPE, "shard results must be [G, N] and outputs [N]");
        if (indices->shape[0] != values->shape[0] || indices->shape[1] != values->shape[1] ||
            out_indices->shape[0] != values->shape[1] || (out_values && out_values->shape[0] != values->shape[1]))
            return fail(CTB_ERR_SHAPE, "shard results and outputs disagree in shape");
        if (indices->dtype != CTB_INT64 || out_indices->dtype != CTB_INT64)
            return fail(CTB_ERR_DTYPE, "indices must be int64");
        if (out_values && out_values->dtype != values->dtype)
            return fail(CTB_ERR_DTYPE, "combined values must have the shards' dtype");
        if (values->dtype == CTB_BFLOAT16) return fail(CTB_ERR_DTYPE, "bfloat16 is not supported");
        if (values->shape[0] > (int64_t(1) << 20)) return fail(CTB_ERR_SHAPE, "too many shards");
        return minmax_combine(op, values, indices, d_row_offsets, out_values, out_indices,
                              static_cast<cudaStream_t>(stream));
    });
}

int ctb_fill_random(const ctb_view* out, int dist, uint64_t seed, uint64_t stream_id,
                    int64_t first_index, double lo, double hi, ctb_stream stream) {
    return guarded([&]() -> int {
        t_error.clear();
        if (int rc = check_views({out})) return rc;
        if (dist != 0 && dist != 1) return fail(CTB_ERR_ARGUMENT, "dist must be 0 (uniform) or 1 (normal)");
        return fill_random(out, dist, seed, stream_id, first_index, lo, hi, static_cast<cudaStream_t>(stream));
    });
}

}  // extern "C"
