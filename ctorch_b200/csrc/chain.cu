// chain.cu — fused two-op chains out = op2(op1(a, b), c) for float32/float64 operands of one
// dtype. The intermediate is rounded to the dtype exactly as the eager pair of binary ops rounds
// it, so the result is bit-identical to ctorch's `op2(op1(a, b), c)` while reading a, b, c once
// and writing out once (no intermediate tensor in HBM).
#include "elementwise.cuh"

namespace ctb {

template <int OP1, int OP2, class T>
int run_chain(const ctb_view* a, const ctb_view* b, const ctb_view* c, const ctb_view* out,
              cudaStream_t st) {
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

int chain_dispatch(int op1, int op2, const ctb_view* a, const ctb_view* b, const ctb_view* c,
                   const ctb_view* out, cudaStream_t st) {
    if (out->dtype == CTB_FLOAT32) return chain_typed<float>(op1, op2, a, b, c, out, st);
    return chain_typed<double>(op1, op2, a, b, c, out, st);
}

}  // namespace ctb
