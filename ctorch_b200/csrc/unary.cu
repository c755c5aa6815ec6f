// unary.cu — neg / abs / relu (int32, int64, float32, float64) and exp / log / sqrt / sigmoid /
// tanh (float32, float64) on the elementwise engine. Semantics of src/ops/functors.h:70-160:
// integer neg/abs wrap through unsigned arithmetic, relu propagates NaN and maps -0.0 to +0.0.
// exp/log/tanh/sigmoid use CUDA's accurate math functions (not bit-identical to the host libm;
// the tests hold them to a few ulp); sqrt is correctly rounded on both sides.
#include "unary.cuh"

namespace ctb {

template <int OP, class T>
int run_unary(const ctb_view* in, const ctb_view* out, cudaStream_t st) {
    constexpr int V = ew_vec<T, T, T, T, 1>();
    const ctb_view* ins[1] = {in};
    const int sizes[2] = {static_cast<int>(sizeof(T)), static_cast<int>(sizeof(T))};
    EwPlan plan;
    const int rc = plan_elementwise(out, ins, 1, sizes, V, plan);
    if (rc) return rc;
    return launch_ew<FnUnary<OP, T>, T, T, T, T, 1>(plan, FnUnary<OP, T>{}, st);
}

template <int OP> int unary_float(const ctb_view* in, const ctb_view* out, cudaStream_t st) {
    if (in->dtype == CTB_FLOAT32) return run_unary<OP, float>(in, out, st);
    return run_unary<OP, double>(in, out, st);
}

template <int OP> int unary_signed(const ctb_view* in, const ctb_view* out, cudaStream_t st) {
    switch (in->dtype) {
    case CTB_FLOAT32: return run_unary<OP, float>(in, out, st);
    case CTB_FLOAT64: return run_unary<OP, double>(in, out, st);
    case CTB_INT32: return run_unary<OP, int32_t>(in, out, st);
    default: return run_unary<OP, int64_t>(in, out, st);
    }
}

// dtypes validated by the caller (capi.cu).
int unary_dispatch(int op, const ctb_view* in, const ctb_view* out, cudaStream_t st) {
    switch (op) {
    case CTB_NEG: return unary_signed<CTB_NEG>(in, out, st);
    case CTB_ABS: return unary_signed<CTB_ABS>(in, out, st);
    case CTB_RELU: return unary_signed<CTB_RELU>(in, out, st);
    case CTB_EXP: return unary_float<CTB_EXP>(in, out, st);
    case CTB_LOG: return unary_float<CTB_LOG>(in, out, st);
    case CTB_SQRT: return unary_float<CTB_SQRT>(in, out, st);
    case CTB_SIGMOID: return unary_float<CTB_SIGMOID>(in, out, st);
    case CTB_TANH: return unary_float<CTB_TANH>(in, out, st);
    }
    return fail(CTB_ERR_ARGUMENT, "unknown unary op");
}

}  // namespace ctb
