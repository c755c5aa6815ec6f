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

// ------------------------------------------------------------------------------------------------
// Combine of a row-sharded max/min over dim 0: G shards' [N] results (values with shard-local row
// indices) into the global result, in rank order with ctorch's rule (the first NaN, otherwise the
// first occurrence of the extreme value, src/ops/reduction_ops_cpu.cpp:236-297). Shard g's rows
// start at global row offs[g], so its local index i is global row offs[g] + i.

template <class T, bool IsMax>
__global__ void minmax_combine_kernel(const T* vals, int64_t vs0, int64_t vs1, const int64_t* idx, int64_t is0,
                                      int64_t is1, const int64_t* offs, int G, int64_t N, T* out_v,
                                      int64_t ov, int64_t* out_i, int64_t oi) {
    dependent_wait();  // the previous kernel in the stream has completed and its writes are visible
    allow_dependents();  // small kernel: the next one in the stream may launch during it
    using R = RMinMax<T, IsMax, true>;
    const int64_t nthr = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t n = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; n < N; n += nthr) {
        typename R::State st = R::init();
        for (int g = 0; g < G; ++g) {
            const typename R::State s{vals[g * vs0 + n * vs1], offs[g] + idx[g * is0 + n * is1]};
            R::combine(st, s);
        }
        if (out_v) out_v[n * ov] = st.v;
        out_i[n * oi] = st.i;
    }
}

int minmax_combine(int op, const ctb_view* values, const ctb_view* indices, const int64_t* d_offsets,
                   const ctb_view* out_values, const ctb_view* out_indices, cudaStream_t st) {
    const int G = static_cast<int>(values->shape[0]);
    const int64_t N = values->shape[1];
    if (N == 0 || G == 0) return CTB_OK;
    const unsigned grid = grid_for((N + 255) / 256, 4);
    const int64_t ov = out_values ? out_values->strides[0] : 0;
#define CTB_MMC(T)                                                                                          \
    {                                                                                                      \
        T* ovp = out_values ? static_cast<T*>(out_values->data) : nullptr;                                 \
        if (op == CTB_MAX)                                                                                 \
            launch_dependent(minmax_combine_kernel<T, true>, grid, 256, 0, st,                                           \
                static_cast<const T*>(values->data), values->strides[0], values->strides[1],               \
                static_cast<const int64_t*>(indices->data), indices->strides[0], indices->strides[1],      \
                d_offsets, G, N, ovp, ov, static_cast<int64_t*>(out_indices->data), out_indices->strides[0]); \
        else                                                                                               \
            launch_dependent(minmax_combine_kernel<T, false>, grid, 256, 0, st,                                          \
                static_cast<const T*>(values->data), values->strides[0], values->strides[1],               \
                static_cast<const int64_t*>(indices->data), indices->strides[0], indices->strides[1],      \
                d_offsets, G, N, ovp, ov, static_cast<int64_t*>(out_indices->data), out_indices->strides[0]); \
        break;                                                                                             \
    }
    switch (values->dtype) {
    case CTB_FLOAT32: CTB_MMC(float)
    case CTB_FLOAT64: CTB_MMC(double)
    case CTB_INT32: CTB_MMC(int32_t)
    case CTB_INT64: CTB_MMC(int64_t)
    case CTB_BOOL: CTB_MMC(uint8_t)
    default: return fail(CTB_ERR_DTYPE, "minmax combine: unsupported dtype");
    }
#undef CTB_MMC
    count_launch();
    return check_launch("minmax_combine");
}

}  // namespace ctb
