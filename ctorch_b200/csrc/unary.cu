// unary.cu — neg / abs / relu (int32, int64, float32, float64) and exp / log / sqrt / sigmoid /
// tanh (float32, float64) on the elementwise engine. Semantics of src/ops/functors.h:70-160:
// integer neg/abs wrap through unsigned arithmetic, relu propagates NaN and maps -0.0 to +0.0.
// exp/log/tanh/sigmoid use CUDA's accurate math functions (not bit-identical to the host libm;
// the tests hold them to a few ulp); sqrt is correctly rounded on both sides.
#include "elementwise.cuh"

namespace ctb {

template <int OP, class T> struct FnUnary {
    __device__ __forceinline__ T operator()(T x) const {
        if constexpr (OP == CTB_RELU) {
            // Selected on the bit pattern so a NaN comes back with its own bits (a float max or
            // compare-select may hand back a canonical NaN instead): positive values and NaNs pass,
            // everything else (including -0.0) becomes +0.0.
            if constexpr (std::is_same_v<T, float>) {
                const uint32_t b = __float_as_uint(x);
                const bool nan = (b & 0x7fffffffu) > 0x7f800000u;
                return __uint_as_float((static_cast<int32_t>(b) > 0 || nan) ? b : 0u);
            } else if constexpr (std::is_same_v<T, double>) {
                const uint64_t b = static_cast<uint64_t>(__double_as_longlong(x));
                const bool nan = (b & 0x7fffffffffffffffULL) > 0x7ff0000000000000ULL;
                return __longlong_as_double(static_cast<long long>((static_cast<int64_t>(b) > 0 || nan) ? b : 0ull));
            } else {
                return x > T(0) ? x : T(0);
            }
        } else if constexpr (OP == CTB_NEG) {
            if constexpr (is_float_v<T>) return -x;
            else return static_cast<T>(std::make_unsigned_t<T>(0) - static_cast<std::make_unsigned_t<T>>(x));
        } else if constexpr (OP == CTB_ABS) {
            if constexpr (std::is_same_v<T, float>) return fabsf(x);
            else if constexpr (std::is_same_v<T, double>) return fabs(x);
            else return x >= T(0) ? x : static_cast<T>(std::make_unsigned_t<T>(0) - static_cast<std::make_unsigned_t<T>>(x));
        } else if constexpr (OP == CTB_EXP) {
            if constexpr (std::is_same_v<T, float>) return expf(x); else return exp(x);
        } else if constexpr (OP == CTB_LOG) {
            if constexpr (std::is_same_v<T, float>) return logf(x); else return log(x);
        } else if constexpr (OP == CTB_SQRT) {
            if constexpr (std::is_same_v<T, float>) return __fsqrt_rn(x); else return __dsqrt_rn(x);
        } else if constexpr (OP == CTB_SIGMOID) {
            if constexpr (std::is_same_v<T, float>) {
                if (x >= 0.0f) return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));
                const float e = expf(x);
                return __fdiv_rn(e, __fadd_rn(1.0f, e));
            } else {
                if (x >= 0.0) return __ddiv_rn(1.0, __dadd_rn(1.0, exp(-x)));
                const double e = exp(x);
                return __ddiv_rn(e, __dadd_rn(1.0, e));
            }
        } else {
            if constexpr (std::is_same_v<T, float>) return tanhf(x); else return tanh(x);
        }
    }
};

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
