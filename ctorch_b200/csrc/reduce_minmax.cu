// reduce_minmax.cu — max / min (values only, any axes) and max / min / argmax / argmin along one
// axis with int64 positions (reducers in reduce.cuh).
#include "reduce.cuh"

namespace ctb {

template <class R>
int run_minmax(const ctb_view* in, const ctb_view* values, const ctb_view* indices, uint32_t mask,
               void* scratch, size_t scratch_bytes, cudaStream_t st, size_t* need_only) {
    RedPlan plan;
    size_t need = 0;
    const ctb_view* first = values ? values : indices;
    const int rc = plan_for<R>(in, first, indices, mask, plan, need);
    if (rc) return rc;
    if (need_only) {
        *need_only = need;
        return CTB_OK;
    }
    plan.args.out = values ? values->data : nullptr;
    return launch_reduction<R>(plan, scratch, scratch_bytes, need, st);
}

template <bool IsMax, bool Indexed>
int minmax_typed(const ctb_view* in, const ctb_view* values, const ctb_view* indices, uint32_t mask,
                 void* scratch, size_t sb, cudaStream_t st, size_t* need_only) {
    switch (in->dtype) {
    case CTB_FLOAT32: return run_minmax<RMinMax<float, IsMax, Indexed>>(in, values, indices, mask, scratch, sb, st, need_only);
    case CTB_FLOAT64: return run_minmax<RMinMax<double, IsMax, Indexed>>(in, values, indices, mask, scratch, sb, st, need_only);
    case CTB_INT32: return run_minmax<RMinMax<int32_t, IsMax, Indexed>>(in, values, indices, mask, scratch, sb, st, need_only);
    case CTB_INT64: return run_minmax<RMinMax<int64_t, IsMax, Indexed>>(in, values, indices, mask, scratch, sb, st, need_only);
    case CTB_BOOL: return run_minmax<RMinMax<uint8_t, IsMax, Indexed>>(in, values, indices, mask, scratch, sb, st, need_only);
    }
    return fail(CTB_ERR_DTYPE, "unsupported reduction dtype");
}

// Values-only max/min over a mask (indices == nullptr) or single-axis with indices.
int minmax_dispatch(int op, const ctb_view* in, const ctb_view* values, const ctb_view* indices,
                    uint32_t mask, void* scratch, size_t sb, cudaStream_t st, size_t* need_only) {
    const bool is_max = op == CTB_MAX;
    if (indices) {
        return is_max ? minmax_typed<true, true>(in, values, indices, mask, scratch, sb, st, need_only)
                      : minmax_typed<false, true>(in, values, indices, mask, scratch, sb, st, need_only);
    }
    return is_max ? minmax_typed<true, false>(in, values, nullptr, mask, scratch, sb, st, need_only)
                  : minmax_typed<false, false>(in, values, nullptr, mask, scratch, sb, st, need_only);
}

}  // namespace ctb
