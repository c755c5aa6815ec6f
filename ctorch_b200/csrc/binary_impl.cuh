// binary_impl.cuh — dtype dispatch for one binary op; instantiated once per op (binary_<op>.cu)
// so the four ops compile in parallel.
#pragma once

#include "elementwise.cuh"

namespace ctb {

template <int OP, class O, class A, class B>
int run_binary(const ctb_view* a, const ctb_view* b, const ctb_view* out, cudaStream_t st) {
    constexpr int V = ew_vec<O, A, B, A, 2>();
    const ctb_view* ins[2] = {a, b};
    const int sizes[3] = {static_cast<int>(sizeof(O)), static_cast<int>(sizeof(A)),
                          static_cast<int>(sizeof(B))};
    EwPlan plan;
    const int rc = plan_elementwise(out, ins, 2, sizes, V, plan);
    if (rc) return rc;
    return launch_ew<FnBinary<OP, O>, O, A, B, A, 2>(plan, FnBinary<OP, O>{}, st);
}

// Operand dtypes are validated by the caller (capi.cu): out == promote(a, b), no bool/bfloat16,
// no integer division.
template <int OP>
int binary_dispatch(const ctb_view* a, const ctb_view* b, const ctb_view* out, cudaStream_t st) {
    const int da = a->dtype, db = b->dtype, dout = out->dtype;
#define CTB_BIN_CASE(DA, DB, DO)                                                               \
    if (da == DA && db == DB && dout == DO)                                                    \
        return run_binary<OP, typename TypeOf<DO>::type, typename TypeOf<DA>::type,            \
                          typename TypeOf<DB>::type>(a, b, out, st);
    if constexpr (OP != CTB_DIV) {
        CTB_BIN_CASE(CTB_INT32, CTB_INT32, CTB_INT32)
        CTB_BIN_CASE(CTB_INT64, CTB_INT64, CTB_INT64)
        CTB_BIN_CASE(CTB_INT32, CTB_INT64, CTB_INT64)
        CTB_BIN_CASE(CTB_INT64, CTB_INT32, CTB_INT64)
    }
    CTB_BIN_CASE(CTB_FLOAT32, CTB_FLOAT32, CTB_FLOAT32)
    CTB_BIN_CASE(CTB_INT32, CTB_FLOAT32, CTB_FLOAT32)
    CTB_BIN_CASE(CTB_FLOAT32, CTB_INT32, CTB_FLOAT32)
    CTB_BIN_CASE(CTB_INT64, CTB_FLOAT32, CTB_FLOAT32)
    CTB_BIN_CASE(CTB_FLOAT32, CTB_INT64, CTB_FLOAT32)
    CTB_BIN_CASE(CTB_FLOAT64, CTB_FLOAT64, CTB_FLOAT64)
    CTB_BIN_CASE(CTB_FLOAT32, CTB_FLOAT64, CTB_FLOAT64)
    CTB_BIN_CASE(CTB_FLOAT64, CTB_FLOAT32, CTB_FLOAT64)
    CTB_BIN_CASE(CTB_INT32, CTB_FLOAT64, CTB_FLOAT64)
    CTB_BIN_CASE(CTB_FLOAT64, CTB_INT32, CTB_FLOAT64)
    CTB_BIN_CASE(CTB_INT64, CTB_FLOAT64, CTB_FLOAT64)
    CTB_BIN_CASE(CTB_FLOAT64, CTB_INT64, CTB_FLOAT64)
#undef CTB_BIN_CASE
    return fail(CTB_ERR_DTYPE, std::string("unsupported dtype combination ") + dtype_name(da) +
                                   ", " + dtype_name(db) + " -> " + dtype_name(dout));
}

}  // namespace ctb
