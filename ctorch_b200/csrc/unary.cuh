// unary.cuh — the unary functors of src/ops/functors.h:70-160 for the elementwise engine, shared by
// ctb_unary (unary.cu) and the binary-then-unary chains (chain_unary.cu).
#pragma once

#include "elementwise.cuh"

namespace ctb {

template <int OP, class T> struct FnUnary {
    // cheap enough per element for the wide row tiles (see ew_rows_long)
    static constexpr bool kWideRows = OP == CTB_RELU || OP == CTB_NEG || OP == CTB_ABS;
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

}  // namespace ctb
