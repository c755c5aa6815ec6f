// chain.cu — fused two-op chains out = op2(op1(a, b), c) for float32/float64 operands of one
// dtype. The intermediate is rounded to the dtype exactly as the eager pair of binary ops rounds
// it, so the result is bit-identical to ctorch's `op2(op1(a, b), c)` while reading a, b, c once
// and writing out once (no intermediate tensor in HBM).
#include "elementwise.cuh"

namespace ctb {

// op2(op1(a, b), b): the chain when its third operand is the second one again, e.g. ctorch's
// (X - r) * r. Read as two inputs, the broadcast row is loaded once per element instead of twice.
template <int OP1, int OP2, class T> struct FnChainRepeat {
    static constexpr bool kWideRows = OP1 != CTB_DIV && OP2 != CTB_DIV;
    __device__ __forceinline__ T operator()(T a, T b) const {
        return BinOp<OP2>::template apply<T>(BinOp<OP1>::template apply<T>(a, b), b);
    }
};

static bool same_view(const ctb_view* x, const ctb_view* y) {
    if (x->data != y->data || x->dtype != y->dtype || x->ndim != y->ndim) return false;
    for (int d = 0; d < x->ndim; ++d)
        if (x->shape[d] != y->shape[d] || x->strides[d] != y->strides[d]) return false;
    return true;
}

template <int OP1, int OP2, class T>
int run_chain(const ctb_view* a, const ctb_view* b, const ctb_view* c, const ctb_view* out,
              cudaStream_t st) {
    if (same_view(b, c)) {
        using Fr = FnChainRepeat<OP1, OP2, T>;
        constexpr int V2 = ew_vec<T, T, T, T, 2>();
        const ctb_view* ins2[2] = {a, b};
        const int sizes2[3] = {static_cast<int>(sizeof(T)), static_cast<int>(sizeof(T)), static_cast<int>(sizeof(T))};
        EwPlan plan2;
        if (int rc = plan_elementwise(out, ins2, 2, sizes2, V2, plan2)) return rc;
        return launch_ew<Fr, T, T, T, T, 2>(plan2, Fr{}, st);
    }
    using Fn = FnChain<OP1, OP2, T, T>;
    constexpr int V = ew_vec<T, T, T, T, 3>();
    const ctb_view* ins[3] = {a, b, c};
    const int sizes[4] = {static_cast<int>(sizeof(T)), static_cast<int>(sizeof(T)),
                          static_cast<int>(sizeof(T)), static_cast<int>(sizeof(T))};
    EwPlan plan;
    const int rc = plan_elementwise(out, ins, 3, sizes, V, plan);
    if (rc) return rc;
    return launch_ew<Fn, T, T, T, T, 3>(plan, Fn{}, st);
}

template <int OP1, class T>
int chain_op2(int op2, const ctb_view* a, const ctb_view* b, const ctb_view* c, const ctb_view* out,
              cudaStream_t st) {
    switch (op2) {
    case CTB_ADD: return run_chain<OP1, CTB_ADD, T>(a, b, c, out, st);
    case CTB_SUB: return run_chain<OP1, CTB_SUB, T>(a, b, c, out, st);
    case CTB_MUL: return run_chain<OP1, CTB_MUL, T>(a, b, c, out, st);
    case CTB_DIV: return run_chain<OP1, CTB_DIV, T>(a, b, c, out, st);
    }
    return fail(CTB_ERR_ARGUMENT, "unknown binary op");
}

template <class T>
int chain_typed(int op1, int op2, const ctb_view* a, const ctb_view* b, const ctb_view* c,
                const ctb_view* out, cudaStream_t st) {
    switch (op1) {
    case CTB_ADD: return chain_op2<CTB_ADD, T>(op2, a, b, c, out, st);
    case CTB_SUB: return chain_op2<CTB_SUB, T>(op2, a, b, c, out, st);
    case CTB_MUL: return chain_op2<CTB_MUL, T>(op2, a, b, c, out, st);
    case CTB_DIV: return chain_op2<CTB_DIV, T>(op2, a, b, c, out, st);
    }
    return fail(CTB_ERR_ARGUMENT, "unknown binary op");
}

int fused_chain_rows(int op1, int op2, const ctb_view* a, const ctb_view* b, const ctb_view* c,
                     const ctb_view* out, cudaStream_t st);  // fused_rows.cu; -1 when it does not apply

int chain_dispatch(int op1, int op2, const ctb_view* a, const ctb_view* b, const ctb_view* c,
                   const ctb_view* out, cudaStream_t st) {
    const int rc = fused_chain_rows(op1, op2, a, b, c, out, st);
    if (rc != -1) return rc;
    if (out->dtype == CTB_FLOAT32) return chain_typed<float>(op1, op2, a, b, c, out, st);
    return chain_typed<double>(op1, op2, a, b, c, out, st);
}

}  // namespace ctb
