// cast.cu — out = in converted to out's dtype (ctb_cast), on the elementwise engine: a strided or
// broadcast source is read in place and written to any layout of out, so a same-dtype cast into a
// contiguous buffer is a strided -> contiguous copy (a CUDA Tensor::contiguous()).
//
// Conversion semantics of ctorch's cast (src/ops/cast_cpu.cpp:21-36): static_cast, with bool read
// as 0/1 and any nonzero (NaN included) written to bool as true. float -> integer truncates
// toward zero; a NaN or out-of-range float -> integer is undefined in C++ (ctorch's x86 build
// gives the integer minimum), and here saturates, NaN giving 0.
#include "elementwise.cuh"

namespace ctb {

template <class D, class S> struct FnCast {
    static constexpr bool kWideRows = true;
    __device__ __forceinline__ D operator()(S x) const {
        if constexpr (std::is_same_v<D, uint8_t> && !std::is_same_v<S, uint8_t>) return x != S(0) ? 1 : 0;
        else return cvt<D>(x);
    }
};

template <class D, class S> int run_cast(const ctb_view* in, const ctb_view* out, cudaStream_t st) {
    constexpr int V = ew_vec<D, S, S, S, 1>();
    const ctb_view* ins[1] = {in};
    const int sizes[2] = {static_cast<int>(sizeof(D)), static_cast<int>(sizeof(S))};
    EwPlan plan;
    const int rc = plan_elementwise(out, ins, 1, sizes, V, plan);
    if (rc) return rc;
    return launch_ew<FnCast<D, S>, D, S, S, S, 1>(plan, FnCast<D, S>{}, st);
}

template <class S> int cast_from(const ctb_view* in, const ctb_view* out, cudaStream_t st) {
    switch (out->dtype) {
    case CTB_FLOAT32: return run_cast<float, S>(in, out, st);
    case CTB_FLOAT64: return run_cast<double, S>(in, out, st);
    case CTB_INT32: return run_cast<int32_t, S>(in, out, st);
    case CTB_INT64: return run_cast<int64_t, S>(in, out, st);
    case CTB_BOOL: return run_cast<uint8_t, S>(in, out, st);
    }
    return fail(CTB_ERR_DTYPE, "cast to bfloat16 not supported");
}

// Dtypes are validated by the caller (capi.cu).
int cast_dispatch(const ctb_view* in, const ctb_view* out, cudaStream_t st) {
    switch (in->dtype) {
    case CTB_FLOAT32: return cast_from<float>(in, out, st);
    case CTB_FLOAT64: return cast_from<double>(in, out, st);
    case CTB_INT32: return cast_from<int32_t>(in, out, st);
    case CTB_INT64: return cast_from<int64_t>(in, out, st);
    case CTB_BOOL: return cast_from<uint8_t>(in, out, st);
    }
    return fail(CTB_ERR_DTYPE, "cast from bfloat16 not supported");
}

}  // namespace ctb
