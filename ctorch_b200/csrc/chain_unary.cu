// chain_unary.cu — out = uop(op(a, b)) in one pass for operands of one dtype, bit-identical to the
// two eager ops (the binary result is rounded to the dtype before the unary op sees it). The
// unary op is relu, neg or abs, e.g. ctorch's relu(add(A, B)) (src/ops/functors.h:49-119) reads
// A and B once and writes the result once instead of writing and re-reading the sum.
#include "unary.cuh"

namespace ctb {

template <int OP, int UOP, class T> struct FnBinUnary {
    static constexpr bool kWideRows = OP != CTB_DIV && FnUnary<UOP, T>::kWideRows;
    __device__ __forceinline__ T operator()(T a, T b) const {
        return FnUnary<UOP, T>{}(BinOp<OP>::template apply<T>(a, b));
    }
};

template <int OP, int UOP, class T>
int run_bin_unary(const ctb_view* a, const ctb_view* b, const ctb_view* out, cudaStream_t st) {
    using Fn = FnBinUnary<OP, UOP, T>;
    constexpr int V = ew_vec<T, T, T, T, 2>();
    const ctb_view* ins[2] = {a, b};
    const int sizes[3] = {static_cast<int>(sizeof(T)), static_cast<int>(sizeof(T)), static_cast<int>(sizeof(T))};
    EwPlan plan;
    const int rc = plan_elementwise(out, ins, 2, sizes, V, plan);
    if (rc) return rc;
    return launch_ew<Fn, T, T, T, T, 2>(plan, Fn{}, st);
}

template <int UOP, class T>
int bin_unary_op(int op, const ctb_view* a, const ctb_view* b, const ctb_view* out, cudaStream_t st) {
    switch (op) {
    case CTB_ADD: return run_bin_unary<CTB_ADD, UOP, T>(a, b, out, st);
    case CTB_SUB: return run_bin_unary<CTB_SUB, UOP, T>(a, b, out, st);
    case CTB_MUL: return run_bin_unary<CTB_MUL, UOP, T>(a, b, out, st);
    case CTB_DIV:
        if constexpr (is_float_v<T>) return run_bin_unary<CTB_DIV, UOP, T>(a, b, out, st);
        break;
    }
    return fail(CTB_ERR_DTYPE, "integer division is not supported; cast operands to float32/float64 first");
}

template <class T>
int bin_unary_typed(int op, int uop, const ctb_view* a, const ctb_view* b, const ctb_view* out, cudaStream_t st) {
    switch (uop) {
    case CTB_RELU: return bin_unary_op<CTB_RELU, T>(op, a, b, out, st);
    case CTB_NEG: return bin_unary_op<CTB_NEG, T>(op, a, b, out, st);
    case CTB_ABS: return bin_unary_op<CTB_ABS, T>(op, a, b, out, st);
    }
    return fail(CTB_ERR_ARGUMENT, "the fused unary op must be relu, neg or abs");
}

// dtypes validated by the caller (capi.cu): a, b, out share one of float32/float64/int32/int64.
int bin_unary_dispatch(int op, int uop, const ctb_view* a, const ctb_view* b, const ctb_view* out,
                       cudaStream_t st) {
    switch (out->dtype) {
    case CTB_FLOAT32: return bin_unary_typed<float>(op, uop, a, b, out, st);
    case CTB_FLOAT64: return bin_unary_typed<double>(op, uop, a, b, out, st);
    case CTB_INT32: return bin_unary_typed<int32_t>(op, uop, a, b, out, st);
    case CTB_INT64: return bin_unary_typed<int64_t>(op, uop, a, b, out, st);
    }
    return fail(CTB_ERR_DTYPE, "unsupported dtype");
}

}  // namespace ctb
