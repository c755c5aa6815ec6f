// reduce_sum.cu — sum / mean / prod dispatch (reducers in reduce.cuh) and the float64 partial
// sums of the multi-GPU whole-tensor sum.
#include "reduce.cuh"

namespace ctb {

template <class R>
int run_reduce(const ctb_view* in, const ctb_view* out, uint32_t mask, void* scratch,
               size_t scratch_bytes, cudaStream_t st, size_t* need_only) {
    RedPlan plan;
    size_t need = 0;
    const int rc = plan_for<R>(in, out, nullptr, mask, plan, need);
    if (rc) return rc;
    if (need_only) {
        *need_only = need;
        return CTB_OK;
    }
    return launch_reduction<R>(plan, scratch, scratch_bytes, need, st);
}

template <bool IsProd>
int accum_dispatch(const ctb_view* in, const ctb_view* out, uint32_t mask, void* scratch,
                   size_t sb, cudaStream_t st, size_t* need_only) {
    switch (in->dtype) {
    case CTB_FLOAT32: return run_reduce<RAccum<float, IsProd>>(in, out, mask, scratch, sb, st, need_only);
    case CTB_FLOAT64: return run_reduce<RAccum<double, IsProd>>(in, out, mask, scratch, sb, st, need_only);
    case CTB_INT32: return run_reduce<RAccum<int32_t, IsProd>>(in, out, mask, scratch, sb, st, need_only);
    case CTB_INT64: return run_reduce<RAccum<int64_t, IsProd>>(in, out, mask, scratch, sb, st, need_only);
    case CTB_BOOL: return run_reduce<RAccum<uint8_t, IsProd>>(in, out, mask, scratch, sb, st, need_only);
    }
    return fail(CTB_ERR_DTYPE, "unsupported reduction dtype");
}

// dtypes validated by the caller (capi.cu).
int sum_like_dispatch(int op, const ctb_view* in, const ctb_view* out, uint32_t mask, void* scratch,
                      size_t sb, cudaStream_t st, size_t* need_only) {
    switch (op) {
    case CTB_SUM: return accum_dispatch<false>(in, out, mask, scratch, sb, st, need_only);
    case CTB_PROD: return accum_dispatch<true>(in, out, mask, scratch, sb, st, need_only);
    case CTB_MEAN:
        if (in->dtype == CTB_FLOAT32) return run_reduce<RMean<float>>(in, out, mask, scratch, sb, st, need_only);
        return run_reduce<RMean<double>>(in, out, mask, scratch, sb, st, need_only);
    }
    return fail(CTB_ERR_ARGUMENT, "unknown reduction op");
}

int sum_partial_dispatch(const ctb_view* in, double* d_partial, void* scratch, size_t sb,
                         cudaStream_t st, size_t* need_only) {
    ctb_view out{};
    out.data = d_partial;
    out.dtype = CTB_FLOAT64;
    out.ndim = 0;
    const uint32_t mask = in->ndim >= 32 ? 0xffffffffu : ((1u << in->ndim) - 1u);
    if (in->dtype == CTB_FLOAT32) return run_reduce<RSumPartial<float>>(in, &out, mask, scratch, sb, st, need_only);
    return run_reduce<RSumPartial<double>>(in, &out, mask, scratch, sb, st, need_only);
}

__global__ void sum_combine_kernel(const double* parts, int n, void* out, int dtype) {
    dependent_wait();  // the previous kernel in the stream has completed and its writes are visible
    allow_dependents();  // small kernel: the next one in the stream may launch during it
    if (blockIdx.x != 0 || threadIdx.x != 0) return;
    double s = 0.0;
    for (int i = 0; i < n; ++i) s = __dadd_rn(s, parts[i]);
    if (dtype == CTB_FLOAT32) *static_cast<float*>(out) = static_cast<float>(s);
    else *static_cast<double*>(out) = s;
}

int sum_combine(const double* parts, int n, const ctb_view* out, cudaStream_t st) {
    launch_dependent(sum_combine_kernel, 1, 32, 0, st, parts, n, out->data, out->dtype);
    count_launch();
    return check_launch("sum_combine");
}

}  // namespace ctb
