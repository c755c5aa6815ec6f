// elementwise.cuh — sm_100a elementwise kernels (binary, unary, fused binary chains).
//
// One functor `Fn` computes an output element from up to three input elements (each in its own
// storage type; Fn converts). The planner (plan.cu) picks one of six launch shapes:
//   Flat      rank 1 after collapsing, unit/zero strides: grid-stride 16-byte packs, 4 in flight
//   RowsLong  unit/zero inner strides, rows >= 1024 packs: CTA tiles of 1024 or 2048 packs along a
//             row, the row's base offsets decoded once per tile (FastDiv, no 64-bit divides)
//   RowsMid   same, rows of 128..1023 packs: warp tiles of 128 packs, decoded once per tile
//   RowsShort same, shorter rows: each pack decodes its own row
//   Tiled     one input read transposed (unit stride on an outer dim): 64x64 tile staged through
//             shared memory so both the transposed read and the output write are coalesced
//   General   anything else: per-element coordinate decode
// Replaces ctorch's one-thread-per-element kernels (src/ops/binary_ops_cuda.cu:53-81,
// src/ops/unary_ops_cuda.cu:50-75), which take a 64-bit div/mod per dim per element.
#pragma once

#include "common.cuh"
#include "plan.cuh"

namespace ctb {

constexpr int kEwBlock = 256;
constexpr int kEwUnroll = 4;
constexpr int kTile = 64;
// Resident CTAs asked of the register allocator for division by a per-row scalar: at 4 (64
// registers) the reciprocal sequence of four packs a thread no longer overlaps its loads, and the
// kernel runs about 40% slower on float32[64,512,1024] / float64[1,512,1].
constexpr int kRowDivMinBlocks = 3;

struct NoIn {};

// Elements per pack: one 16-byte chunk of the narrowest operand, capped so the widest operand's
// pack stays within 32 bytes (a bool <- int64 cast takes 4 elements, not 16).
template <class O, class I0, class I1, class I2, int NIN> constexpr int ew_vec() {
    int m = sizeof(O), w = sizeof(O);
    if ((int)sizeof(I0) < m) m = sizeof(I0);
    if ((int)sizeof(I0) > w) w = sizeof(I0);
    if (NIN > 1 && (int)sizeof(I1) < m) m = sizeof(I1);
    if (NIN > 1 && (int)sizeof(I1) > w) w = sizeof(I1);
    if (NIN > 2 && (int)sizeof(I2) < m) m = sizeof(I2);
    if (NIN > 2 && (int)sizeof(I2) > w) w = sizeof(I2);
    const int v = 16 / m;
    return v * w > 32 ? 32 / w : v;
}

template <class Fn, class O, class I0, class I1, class I2, int NIN>
__device__ __forceinline__ O ew_apply(const Fn& fn, I0 x0, I1 x1, I2 x2) {
    if constexpr (NIN == 1) return fn(x0);
    else if constexpr (NIN == 2) return fn(x0, x1);
    else return fn(x0, x1, x2);
}

// Row base offsets for each operand: decode `row` over dims [0, rank-2] (outermost first).
__device__ __forceinline__ void ew_decode_row(const EwArgs& p, uint64_t row, int nops,
                                              int64_t* off) {
    for (int o = 0; o < kMaxOps; ++o) off[o] = 0;
    for (int d = p.rank - 2; d >= 0; --d) {
        uint64_t q, r;
        p.div[d].divmod(row, q, r);
        for (int o = 0; o < nops; ++o) off[o] += static_cast<int64_t>(r) * p.stride[o][d];
        row = q;
    }
}

// Division by a divisor that is constant along a row, from its correctly rounded reciprocal
// y = RN(1/b), computed once per row:
//   q0 = RN(a*y)                   within about 2 ulp of a/b
//   q1 = RN(q0 + RN(a - b*q0)*y)   faithful (one of the two neighbours of a/b)
//   q2 = RN(q1 + (a - b*q1)*y)     = RN(a/b)
// a - b*q1 is exact in an FMA because q1 is faithful, and the last step is Markstein's theorem
// (P. Markstein, IBM J. Res. Dev. 34(1), 1990): with y within half an ulp of 1/b and q1 faithful,
// q1 + r*y cannot land on the other side of a rounding midpoint from a/b. The theorem assumes no
// overflow, underflow or subnormal along the way, so the sequence only runs when a, b and the
// quotient have exponents at least `kMargin` away from both ends of the range; zeros,
// infinities, NaNs, subnormals and extreme magnitudes take the IEEE division. Either way the
// result is the correctly rounded quotient, bit-identical to a / b.
template <class T> struct FpTraits;
template <> struct FpTraits<double> {
    static constexpr int kMax = 2046, kMargin = 64, kBias = 1023;
};
template <> struct FpTraits<float> {
    static constexpr int kMax = 254, kMargin = 32, kBias = 127;
};

template <class T> __device__ __forceinline__ int fp_exponent(T x) {
    if constexpr (std::is_same_v<T, double>)
        return static_cast<int>((static_cast<unsigned>(__double2hiint(x)) >> 20) & 0x7ff);
    else
        return static_cast<int>((__float_as_uint(x) >> 23) & 0xff);
}

// The per-row state: the divisor, its reciprocal, and the range [lo, lo + span] of dividend
// exponents for which the sequence runs. A divisor that is itself out of range gets lo = 2^30,
// span = 0, a range no exponent (0..2047) falls in.
template <class T> struct RowDivisor {
    T b, y;
    int lo;
    unsigned span;
};

template <class T> __device__ __forceinline__ RowDivisor<T> row_divisor(T b) {
    using F = FpTraits<T>;
    RowDivisor<T> d;
    d.b = b;
    const int eb = fp_exponent(b);
    // quotient exponent ea - eb + bias must also stay in [margin, max - margin]
    const int lo = max(F::kMargin, eb - F::kBias + F::kMargin);
    const int hi = min(F::kMax - F::kMargin, eb - F::kBias + F::kMax - F::kMargin);
    const bool ok = eb >= F::kMargin && eb <= F::kMax - F::kMargin && hi >= lo;
    d.lo = ok ? lo : (1 << 30);
    d.span = ok ? static_cast<unsigned>(hi - lo) : 0u;
    if constexpr (std::is_same_v<T, double>) d.y = ok ? __drcp_rn(b) : 0.0;
    else d.y = ok ? __frcp_rn(b) : 0.0f;
    return d;
}

template <class T> __device__ __forceinline__ T div_by_row(T a, const RowDivisor<T>& d) {
    if (static_cast<unsigned>(fp_exponent(a) - d.lo) <= d.span) {
        if constexpr (std::is_same_v<T, double>) {
            const double q0 = __dmul_rn(a, d.y);
            const double q1 = __fma_rn(__fma_rn(-d.b, q0, a), d.y, q0);
            return __fma_rn(__fma_rn(-d.b, q1, a), d.y, q1);
        } else {
            const float q0 = __fmul_rn(a, d.y);
            const float q1 = __fmaf_rn(__fmaf_rn(-d.b, q0, a), d.y, q0);
            return __fmaf_rn(__fmaf_rn(-d.b, q1, a), d.y, q1);
        }
    }
    return BinOp<CTB_DIV>::template apply<T>(a, d.b);
}

// kWideRows: cheap enough per element for the wide row tiles (see ew_rows_long); division is not.
template <int OP, class O> struct FnBinary {
    static constexpr bool kWideRows = OP != CTB_DIV;
    template <class A, class B> __device__ __forceinline__ O operator()(A a, B b) const {
        return BinOp<OP>::template apply<O>(cvt<O>(a), cvt<O>(b));
    }
};

// Row kernels whose second operand is a per-row scalar check RowPrep<Fn>::kActive: when it is set
// (float and double division) they prepare the scalar once per row with row_divisor and divide each
// element of the row with div_by_row; every other functor is applied as it is.
template <class Fn> struct RowPrep {
    static constexpr bool kActive = false;
};
template <class O> struct RowPrep<FnBinary<CTB_DIV, O>> {
    static constexpr bool kActive = is_float_v<O>;
};

// ------------------------------------------------------------------------------------------------
template <class Fn, class O, class I0, class I1, class I2, int NIN>
__global__ void __launch_bounds__(kEwBlock) ew_flat(EwArgs p, Fn fn) {
    dependent_wait();  // the previous kernel in the stream has completed and its writes are visible
    constexpr int V = ew_vec<O, I0, I1, I2, NIN>();
    constexpr int U = kEwUnroll;
    O* __restrict__ out = static_cast<O*>(p.out);
    const I0* __restrict__ in0 = static_cast<const I0*>(p.in[0]);
    const I1* __restrict__ in1 = static_cast<const I1*>(p.in[1]);
    const I2* __restrict__ in2 = static_cast<const I2*>(p.in[2]);
    const bool b0 = p.stride[1][0] == 0;
    const bool b1 = NIN > 1 && p.stride[2][0] == 0;
    const bool b2 = NIN > 2 && p.stride[3][0] == 0;
    const I0 s0 = b0 ? in0[0] : I0{};
    I1 s1{};
    I2 s2{};
    if constexpr (NIN > 1) s1 = b1 ? in1[0] : I1{};
    if constexpr (NIN > 2) s2 = b2 ? in2[0] : I2{};

    const int64_t n = p.n;
    const int64_t nvec = n / V;
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nthr = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t base = tid; base < nvec; base += nthr * U) {
        Pack<I0, V> x0[U];
        Pack<I1, V> x1[U];
        Pack<I2, V> x2[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t v = base + u * nthr;
            if (v < nvec) {
                if (!b0) x0[u] = load_pack<I0, V>(in0 + v * V);
                if constexpr (NIN > 1) if (!b1) x1[u] = load_pack<I1, V>(in1 + v * V);
                if constexpr (NIN > 2) if (!b2) x2[u] = load_pack<I2, V>(in2 + v * V);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t v = base + u * nthr;
            if (v < nvec) {
                Pack<O, V> o;
#pragma unroll
                for (int e = 0; e < V; ++e)
                    o.v[e] = ew_apply<Fn, O, I0, I1, I2, NIN>(fn, b0 ? s0 : x0[u].v[e],
                                                              b1 ? s1 : x1[u].v[e],
                                                              b2 ? s2 : x2[u].v[e]);
                store_pack<O, V>(out + v * V, o);
            }
        }
    }
    for (int64_t i = nvec * V + tid; i < n; i += nthr) {
        out[i] = ew_apply<Fn, O, I0, I1, I2, NIN>(fn, in0[b0 ? 0 : i], NIN > 1 ? in1[b1 ? 0 : i] : I1{},
                                                  NIN > 2 ? in2[b2 ? 0 : i] : I2{});
    }
    allow_dependents();  // the next kernel in the stream may launch while this one winds down
}

// ------------------------------------------------------------------------------------------------
// Which inputs are constant along the inner dim (stride 0): bit i for input i. BMASK >= 0 fixes it
// at compile time, so a per-row scalar operand holds one register instead of a pack's worth;
// BMASK < 0 reads it from the strides at run time.
template <int BMASK, int NIN>
__device__ __forceinline__ void inner_bcast(const EwArgs& p, bool& b0, bool& b1, bool& b2) {
    const int r = p.rank - 1;
    if constexpr (BMASK >= 0) {
        b0 = BMASK & 1;
        b1 = NIN > 1 && (BMASK & 2);
        b2 = NIN > 2 && (BMASK & 4);
    } else {
        b0 = p.stride[1][r] == 0;
        b1 = NIN > 1 && p.stride[2][r] == 0;
        b2 = NIN > 2 && p.stride[3][r] == 0;
    }
}

template <class Fn, class O, class I0, class I1, class I2, int NIN, int BMASK, int U = kEwUnroll>
__device__ __forceinline__ void ew_row_segment(const EwArgs& p, const Fn& fn, const int64_t* off,
                                               int64_t c0, int64_t cstep, int count) {
    constexpr int V = ew_vec<O, I0, I1, I2, NIN>();
    O* __restrict__ out = static_cast<O*>(p.out) + off[0];
    const I0* __restrict__ in0 = static_cast<const I0*>(p.in[0]) + off[1];
    const I1* __restrict__ in1 = static_cast<const I1*>(p.in[1]) + off[2];
    const I2* __restrict__ in2 = static_cast<const I2*>(p.in[2]) + off[3];
    bool b0, b1, b2;
    inner_bcast<BMASK, NIN>(p, b0, b1, b2);
    const I0 s0 = b0 ? in0[0] : I0{};
    I1 s1{};
    I2 s2{};
    if constexpr (NIN > 1) s1 = b1 ? in1[0] : I1{};
    if constexpr (NIN > 2) s2 = b2 ? in2[0] : I2{};
    Pack<I0, V> x0[U];
    Pack<I1, V> x1[U];
    Pack<I2, V> x2[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int64_t c = c0 + u * cstep;
        if (u < count && c < p.vpr) {
            if (!b0) x0[u] = load_pack<I0, V>(in0 + c * V);
            if constexpr (NIN > 1) if (!b1) x1[u] = load_pack<I1, V>(in1 + c * V);
            if constexpr (NIN > 2) if (!b2) x2[u] = load_pack<I2, V>(in2 + c * V);
        }
    }
    if constexpr (BMASK == 2 && NIN == 2 && RowPrep<Fn>::kActive) {
        const RowDivisor<O> d = row_divisor<O>(cvt<O>(s1));
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t c = c0 + u * cstep;
            if (u < count && c < p.vpr) {
                Pack<O, V> o;
#pragma unroll
                for (int e = 0; e < V; ++e) o.v[e] = div_by_row<O>(cvt<O>(x0[u].v[e]), d);
                store_pack_split<O, V>(out + c * V, o);
            }
        }
    } else {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t c = c0 + u * cstep;
            if (u < count && c < p.vpr) {
                Pack<O, V> o;
#pragma unroll
                for (int e = 0; e < V; ++e)
                    o.v[e] = ew_apply<Fn, O, I0, I1, I2, NIN>(fn, b0 ? s0 : x0[u].v[e],
                                                              b1 ? s1 : x1[u].v[e],
                                                              b2 ? s2 : x2[u].v[e]);
                store_pack<O, V>(out + c * V, o);
            }
        }
    }
}

// Min resident CTAs to ask of the register allocator: 4 when the packs live across the load
// latency are small (<= 48 bytes per thread-pack; 3 with three inputs), else 2.
template <class O, class I0, class I1, class I2, int NIN, int BMASK> constexpr int rows_min_blocks() {
    constexpr int V = ew_vec<O, I0, I1, I2, NIN>();
    if (BMASK < 0) return 2;
    int bytes = V * static_cast<int>(sizeof(O));
    if (!(BMASK & 1)) bytes += V * static_cast<int>(sizeof(I0));
    if (NIN > 1 && !(BMASK & 2)) bytes += V * static_cast<int>(sizeof(I1));
    if (NIN > 2 && !(BMASK & 4)) bytes += V * static_cast<int>(sizeof(I2));
    // three inputs with one of them a per-row scalar still carry a scalar per pack in flight
    if (NIN > 2 && bytes <= 48) return 3;
    return bytes <= 48 ? 4 : 2;
}

// Rows of at least kRowsLongPacks packs: CTA tiles of kEwBlock x U packs along one row, the row's
// base offsets decoded once per tile; p.aux holds the tiles per row for that U. The launcher
// takes U = 4, or 8 with half the resident CTAs on rows of 2048 packs or more (one tile covers a
// whole 8192-float row: about 5% faster there than two tiles of 4 packs a thread).
template <class Fn, class O, class I0, class I1, class I2, int NIN, int BMASK, int U, int MINB>
__global__ void __launch_bounds__(kEwBlock, MINB) ew_rows_long(EwArgs p, Fn fn) {
    dependent_wait();  // the previous kernel in the stream has completed and its writes are visible
    const int64_t seg = static_cast<int64_t>(kEwBlock) * U;
    const int64_t tiles = p.rows * static_cast<int64_t>(p.aux.d);
    for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
        uint64_t row, s;
        p.aux.divmod(static_cast<uint64_t>(t), row, s);
        int64_t off[kMaxOps];
        ew_decode_row(p, row, NIN + 1, off);
        ew_row_segment<Fn, O, I0, I1, I2, NIN, BMASK, U>(p, fn, off, static_cast<int64_t>(s) * seg + threadIdx.x,
                                                         kEwBlock, U);
    }
    allow_dependents();  // the next kernel in the stream may launch while this one winds down
}

// Rows of kRowsMidPacks up to kRowsLongPacks packs: each warp takes tiles of 32 x U packs along
// one row, so the row's base offsets (and a per-row divisor) are worked out once per tile rather
// than per pack. p.aux holds the tiles per row for that U.
template <class Fn, class O, class I0, class I1, class I2, int NIN, int BMASK, int U, int MINB>
__global__ void __launch_bounds__(kEwBlock, MINB) ew_rows_mid(EwArgs p, Fn fn) {
    dependent_wait();  // the previous kernel in the stream has completed and its writes are visible
    constexpr int kWarps = kEwBlock / 32;
    const int64_t seg = 32 * U;
    const int64_t tiles = p.rows * static_cast<int64_t>(p.aux.d);
    const int64_t nw = static_cast<int64_t>(gridDim.x) * kWarps;
    const int lane = threadIdx.x & 31;
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5); t < tiles; t += nw) {
        uint64_t row, s;
        p.aux.divmod(static_cast<uint64_t>(t), row, s);
        int64_t off[kMaxOps];
        ew_decode_row(p, row, NIN + 1, off);
        ew_row_segment<Fn, O, I0, I1, I2, NIN, BMASK, U>(p, fn, off, static_cast<int64_t>(s) * seg + lane, 32, U);
    }
    allow_dependents();  // the next kernel in the stream may launch while this one winds down
}

template <class Fn, class O, class I0, class I1, class I2, int NIN, int BMASK, int MINB>
__global__ void __launch_bounds__(kEwBlock, MINB) ew_rows_short(EwArgs p, Fn fn) {
    dependent_wait();  // the previous kernel in the stream has completed and its writes are visible
    constexpr int V = ew_vec<O, I0, I1, I2, NIN>();
    constexpr int U = kEwUnroll;
    bool b0, b1, b2;
    inner_bcast<BMASK, NIN>(p, b0, b1, b2);
    O* __restrict__ out = static_cast<O*>(p.out);
    const I0* __restrict__ in0 = static_cast<const I0*>(p.in[0]);
    const I1* __restrict__ in1 = static_cast<const I1*>(p.in[1]);
    const I2* __restrict__ in2 = static_cast<const I2*>(p.in[2]);
    const int64_t nvec = p.rows * p.vpr;
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nthr = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t base = tid; base < nvec; base += nthr * U) {
        int64_t oo[U];
        Pack<I0, V> x0[U];
        Pack<I1, V> x1[U];
        Pack<I2, V> x2[U];
        I0 s0[U];
        I1 s1[U];
        I2 s2[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t v = base + u * nthr;
            oo[u] = -1;
            if (v < nvec) {
                uint64_t row, c;
                p.aux.divmod(static_cast<uint64_t>(v), row, c);
                int64_t off[kMaxOps];
                ew_decode_row(p, row, NIN + 1, off);
                const int64_t cv = static_cast<int64_t>(c) * V;
                oo[u] = off[0] + cv;
                if (b0) s0[u] = in0[off[1]];
                else x0[u] = load_pack<I0, V>(in0 + off[1] + cv);
                if constexpr (NIN > 1) {
                    if (b1) s1[u] = in1[off[2]];
                    else x1[u] = load_pack<I1, V>(in1 + off[2] + cv);
                }
                if constexpr (NIN > 2) {
                    if (b2) s2[u] = in2[off[3]];
                    else x2[u] = load_pack<I2, V>(in2 + off[3] + cv);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (oo[u] >= 0) {
                Pack<O, V> o;
                if constexpr (BMASK == 2 && NIN == 2 && RowPrep<Fn>::kActive) {
                    const RowDivisor<O> d = row_divisor<O>(cvt<O>(s1[u]));
#pragma unroll
                    for (int e = 0; e < V; ++e) o.v[e] = div_by_row<O>(cvt<O>(x0[u].v[e]), d);
                    store_pack_split<O, V>(out + oo[u], o);
                } else {
#pragma unroll
                    for (int e = 0; e < V; ++e)
                        o.v[e] = ew_apply<Fn, O, I0, I1, I2, NIN>(fn, b0 ? s0[u] : x0[u].v[e],
                                                                  b1 ? s1[u] : x1[u].v[e],
                                                                  b2 ? s2[u] : x2[u].v[e]);
                    store_pack<O, V>(out + oo[u], o);
                }
            }
        }
    }
    allow_dependents();  // the next kernel in the stream may launch while this one winds down
}

// ------------------------------------------------------------------------------------------------
template <class Fn, class O, class I0, class I1, class I2, int NIN>
__global__ void __launch_bounds__(kEwBlock) ew_general(EwArgs p, Fn fn) {
    dependent_wait();  // the previous kernel in the stream has completed and its writes are visible
    O* __restrict__ out = static_cast<O*>(p.out);
    const I0* __restrict__ in0 = static_cast<const I0*>(p.in[0]);
    const I1* __restrict__ in1 = static_cast<const I1*>(p.in[1]);
    const I2* __restrict__ in2 = static_cast<const I2*>(p.in[2]);
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nthr = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = tid; i < p.n; i += nthr) {
        uint64_t rem = static_cast<uint64_t>(i);
        int64_t off[kMaxOps] = {0, 0, 0, 0};
        for (int d = p.rank - 1; d >= 0; --d) {
            uint64_t q, c;
            p.div[d].divmod(rem, q, c);
#pragma unroll
            for (int o = 0; o <= NIN; ++o) off[o] += static_cast<int64_t>(c) * p.stride[o][d];
            rem = q;
        }
        out[off[0]] = ew_apply<Fn, O, I0, I1, I2, NIN>(fn, in0[off[1]], NIN > 1 ? in1[off[2]] : I1{},
                                                       NIN > 2 ? in2[off[3]] : I2{});
    }
    allow_dependents();  // the next kernel in the stream may launch while this one winds down
}

// ------------------------------------------------------------------------------------------------
// Tiled: binary op where input XOP (1 or 2) has unit stride on dim p.pdim instead of the inner
// dim. Each CTA stages a 64(p) x 64(l) tile of that input in shared memory, reading it along p
// (coalesced), then writes output rows along l (coalesced).
template <class Fn, class O, class I0, class I1, int XOP>
__global__ void __launch_bounds__(kEwBlock) ew_tiled(EwArgs p, Fn fn) {
    dependent_wait();  // the previous kernel in the stream has completed and its writes are visible
    using X = std::conditional_t<XOP == 1, I0, I1>;
    using Y = std::conditional_t<XOP == 1, I1, I0>;
    constexpr int YOP = XOP == 1 ? 2 : 1;
    __shared__ X tile[kTile][kTile + 1];
    const int r = p.rank - 1;
    const int pd = p.pdim;
    const int64_t L = p.shape[r];
    const int64_t P = p.shape[pd];
    const int64_t sXl = p.stride[XOP][r];
    const int64_t sYl = p.stride[YOP][r];
    const int64_t sYp = p.stride[YOP][pd];
    const int64_t sOp = p.stride[0][pd];
    const X* __restrict__ xin = static_cast<const X*>(p.in[XOP - 1]);
    const Y* __restrict__ yin = static_cast<const Y*>(p.in[YOP - 1]);
    O* __restrict__ out = static_cast<O*>(p.out);
    const int64_t tiles_l = static_cast<int64_t>(p.aux.d);
    const int64_t tiles_p = static_cast<int64_t>(p.aux2.d);
    const int64_t total = (p.n / (L * P)) * tiles_l * tiles_p;
    for (int64_t t = blockIdx.x; t < total; t += gridDim.x) {
        uint64_t rest, tl, batch, tp;
        p.aux.divmod(static_cast<uint64_t>(t), rest, tl);
        p.aux2.divmod(rest, batch, tp);
        int64_t offO = 0, offX = 0, offY = 0;
        for (int d = r - 1; d >= 0; --d) {
            if (d == pd) continue;
            uint64_t q, c;
            p.div[d].divmod(batch, q, c);
            offO += static_cast<int64_t>(c) * p.stride[0][d];
            offX += static_cast<int64_t>(c) * p.stride[XOP][d];
            offY += static_cast<int64_t>(c) * p.stride[YOP][d];
            batch = q;
        }
        const int64_t l0 = static_cast<int64_t>(tl) * kTile;
        const int64_t p0 = static_cast<int64_t>(tp) * kTile;
        constexpr int kPer = kTile * kTile / kEwBlock;
        // issue every global load of the tile (transposed input and the row-major operand) before
        // the barrier, so both latencies overlap
        X xr[kPer];
        Y yr[kPer];
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int k = threadIdx.x + j * kEwBlock;
            const int li = k >> 6, pi = k & 63;
            const int64_t pp = p0 + pi, ll = l0 + li;
            if (pp < P && ll < L) xr[j] = xin[offX + pp + ll * sXl];
        }
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int k = threadIdx.x + j * kEwBlock;
            const int pi = k >> 6, li = k & 63;
            const int64_t pp = p0 + pi, ll = l0 + li;
            if (pp < P && ll < L) yr[j] = yin[offY + pp * sYp + ll * sYl];
        }
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int k = threadIdx.x + j * kEwBlock;
            tile[k >> 6][k & 63] = xr[j];
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int k = threadIdx.x + j * kEwBlock;
            const int pi = k >> 6, li = k & 63;
            const int64_t pp = p0 + pi, ll = l0 + li;
            if (pp < P && ll < L) {
                const X x = tile[li][pi];
                O o;
                if constexpr (XOP == 1) o = fn(x, yr[j]);
                else o = fn(yr[j], x);
                out[offO + pp * sOp + ll] = o;
            }
        }
        __syncthreads();
    }
    allow_dependents();  // the next kernel in the stream may launch while this one winds down
}

// Tiled with 4-element packs: the transposed input is read as packs of 4 along its unit-stride
// dim p, the other input and the output as packs of 4 along the inner dim l, so a 64x64 tile costs
// each thread 4 pack loads of each input and 4 pack stores. Edge tiles fall back to elements.
// Requires (checked on the host, EwArgs::tiled_vec): pack-aligned bases and every stride other than
// the unit ones a multiple of 4 elements; the row-major input has unit inner stride.
// TL: the tile's extent along l (the output's and the row-major operand's unit-stride dim), 64 or
// 128; the CTA has TL / 64 x 256 threads, each moving 4 packs of each operand per tile. With
// TL = 128 the row-major operand and the output move in 512-byte runs instead of 256 (DRAM reads
// of 256-byte runs spaced a row apart are ~10% slower) at the same bytes in flight per thread.
template <class Fn, class O, class I0, class I1, int XOP, int TL = kTile>
__global__ void __launch_bounds__(TL / kTile * kEwBlock) ew_tiled4(EwArgs p, Fn fn) {
    dependent_wait();  // the previous kernel in the stream has completed and its writes are visible
    using X = std::conditional_t<XOP == 1, I0, I1>;
    using Y = std::conditional_t<XOP == 1, I1, I0>;
    constexpr int YOP = XOP == 1 ? 2 : 1;
    constexpr int TP = kTile;
    constexpr int NT = TL / kTile * kEwBlock;
    constexpr int kPer = TL * TP / 4 / NT;  // packs per thread (4)
    __shared__ X tile[TL][TP + 1];
    const int r = p.rank - 1;
    const int pd = p.pdim;
    const int64_t L = p.shape[r];
    const int64_t P = p.shape[pd];
    const int64_t sXl = p.stride[XOP][r];
    const int64_t sYp = p.stride[YOP][pd];
    const int64_t sOp = p.stride[0][pd];
    const X* __restrict__ xin = static_cast<const X*>(p.in[XOP - 1]);
    const Y* __restrict__ yin = static_cast<const Y*>(p.in[YOP - 1]);
    O* __restrict__ out = static_cast<O*>(p.out);
    const int64_t tiles_l = static_cast<int64_t>(p.aux.d);
    const int64_t tiles_p = static_cast<int64_t>(p.aux2.d);
    const int64_t total = (p.n / (L * P)) * tiles_l * tiles_p;
    for (int64_t t = blockIdx.x; t < total; t += gridDim.x) {
        uint64_t rest, tl, batch, tp;
        p.aux.divmod(static_cast<uint64_t>(t), rest, tl);
        p.aux2.divmod(rest, batch, tp);
        int64_t offO = 0, offX = 0, offY = 0;
        for (int d = r - 1; d >= 0; --d) {
            if (d == pd) continue;
            uint64_t q, c;
            p.div[d].divmod(batch, q, c);
            offO += static_cast<int64_t>(c) * p.stride[0][d];
            offX += static_cast<int64_t>(c) * p.stride[XOP][d];
            offY += static_cast<int64_t>(c) * p.stride[YOP][d];
            batch = q;
        }
        const int64_t l0 = static_cast<int64_t>(tl) * TL;
        const int64_t p0 = static_cast<int64_t>(tp) * TP;
        const bool full = p0 + TP <= P && l0 + TL <= L;
        if (full) {
            const X* xt = xin + offX + p0 + l0 * sXl;
            const Y* yt = yin + offY + p0 * sYp + l0;
            O* ot = out + offO + p0 * sOp + l0;
            Pack<X, 4> xr[kPer];
            Pack<Y, 4> yr[kPer];
#pragma unroll
            for (int j = 0; j < kPer; ++j) {
                const int k = threadIdx.x + j * NT;
                const int li = k / (TP / 4), pg = k % (TP / 4);  // X: pack pg of row li (along p)
                xr[j] = load_pack<X, 4>(xt + 4 * pg + li * sXl);
            }
#pragma unroll
            for (int j = 0; j < kPer; ++j) {
                const int k = threadIdx.x + j * NT;
                const int pi = k / (TL / 4), lg = k % (TL / 4);  // Y: pack lg of row pi (along l)
                yr[j] = load_pack<Y, 4>(yt + pi * sYp + 4 * lg);
            }
#pragma unroll
            for (int j = 0; j < kPer; ++j) {
                const int k = threadIdx.x + j * NT;
                const int li = k / (TP / 4), pg = k % (TP / 4);
#pragma unroll
                for (int e = 0; e < 4; ++e) tile[li][4 * pg + e] = xr[j].v[e];
            }
            __syncthreads();
#pragma unroll
            for (int j = 0; j < kPer; ++j) {
                const int k = threadIdx.x + j * NT;
                const int pi = k / (TL / 4), lg = k % (TL / 4);
                Pack<O, 4> o;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const X x = tile[4 * lg + e][pi];
                    if constexpr (XOP == 1) o.v[e] = fn(x, yr[j].v[e]);
                    else o.v[e] = fn(yr[j].v[e], x);
                }
                store_pack<O, 4>(ot + pi * sOp + 4 * lg, o);
            }
            __syncthreads();
        } else {
            for (int k = threadIdx.x; k < TL * TP; k += NT) {
                const int li = k / TP, pi = k % TP;
                const int64_t pp = p0 + pi, ll = l0 + li;
                if (pp < P && ll < L) tile[li][pi] = xin[offX + pp + ll * sXl];
            }
            __syncthreads();
            for (int k = threadIdx.x; k < TL * TP; k += NT) {
                const int pi = k / TL, li = k % TL;
                const int64_t pp = p0 + pi, ll = l0 + li;
                if (pp < P && ll < L) {
                    const X x = tile[li][pi];
                    const Y y = yin[offY + pp * sYp + ll];
                    O o;
                    if constexpr (XOP == 1) o = fn(x, y);
                    else o = fn(y, x);
                    out[offO + pp * sOp + ll] = o;
                }
            }
            __syncthreads();
        }
    }
    allow_dependents();  // the next kernel in the stream may launch while this one winds down
}

// ------------------------------------------------------------------------------------------------
// Launcher. Returns a ctb_status.

// One wave of resident CTAs of `kernel` (grid-stride loops cover the rest): no tail of a partly
// filled second wave.
template <class K> inline unsigned wave_grid(K kernel, int64_t work) {
    const int64_t slots = static_cast<int64_t>(sm_count()) *
                          resident_ctas(reinterpret_cast<const void*>(kernel), kEwBlock);
    const int64_t g = work < slots ? work : slots;
    return static_cast<unsigned>(g < 1 ? 1 : g);
}

// Bit i set when input i has stride 0 along the inner dim.
inline int inner_mask(const EwArgs& a, int nin) {
    int m = 0;
    for (int i = 0; i < nin; ++i)
        if (a.stride[1 + i][a.rank - 1] == 0) m |= 1 << i;
    return m;
}

template <class Fn, class O, class I0, class I1 = I0, class I2 = I0, int NIN = 1>
int launch_ew(const EwPlan& plan, Fn fn, cudaStream_t st) {
    constexpr int V = ew_vec<O, I0, I1, I2, NIN>();
    const EwArgs& a = plan.args;
    switch (plan.path) {
    case EwPath::Empty:
        return CTB_OK;
    case EwPath::Flat: {
        const int64_t nvec = a.n / V;
        const int64_t work = (nvec + kEwBlock * kEwUnroll - 1) / (kEwBlock * kEwUnroll);
        auto k = &ew_flat<Fn, O, I0, I1, I2, NIN>;
        launch_dependent(k, wave_grid(k, work), kEwBlock, 0, st, a, fn);
        break;
    }
    case EwPath::RowsLong: {
        // wide tiles only for 4-byte types throughout (mixed widths double the registers a pack
        // takes, and 8-byte types spill at 8 packs a thread)
        constexpr bool kWide = Fn::kWideRows && sizeof(O) == 4 && sizeof(I0) == 4 &&
                               (NIN < 2 || sizeof(I1) == 4) && (NIN < 3 || sizeof(I2) == 4);
        const bool wide = kWide && a.vpr >= 2 * kRowsLongPacks;
        EwArgs al = a;
        const int64_t seg = static_cast<int64_t>(kEwBlock) * (wide ? 8 : 4);
        al.aux = FastDiv(static_cast<uint64_t>((a.vpr + seg - 1) / seg));
        const int64_t tiles = a.rows * static_cast<int64_t>(al.aux.d);
#define CTB_RL(M, U, B)                                                  \
    {                                                                    \
        auto k = &ew_rows_long<Fn, O, I0, I1, I2, NIN, M, U, B>;         \
        launch_dependent(k, wave_grid(k, tiles), kEwBlock, 0, st, al, fn);             \
    }
#define CTB_RL2(M)                                                       \
    if constexpr (kWide) {                                               \
        if (wide) CTB_RL(M, 8, 2)                                        \
        else CTB_RL(M, 4, (rows_min_blocks<O, I0, I1, I2, NIN, M>()))    \
    } else {                                                             \
        CTB_RL(M, 4, (rows_min_blocks<O, I0, I1, I2, NIN, M>()))         \
    }
        switch (inner_mask(a, NIN)) {
        case 0: CTB_RL2(0) break;
        case 1: CTB_RL2(1) break;
        case 2:
            if constexpr (NIN > 1) {
                // division by a per-row scalar: tiles of 4 packs a thread at kRowDivMinBlocks
                if constexpr (RowPrep<Fn>::kActive) {
                    CTB_RL(2, 4, kRowDivMinBlocks)
                } else {
                    CTB_RL2(2)
                }
                break;
            }
            [[fallthrough]];
        default: CTB_RL(-1, 4, 2) break;
        }
#undef CTB_RL2
#undef CTB_RL
        break;
    }
    case EwPath::RowsMid: {
        const int64_t tiles = a.rows * static_cast<int64_t>(a.aux.d);
        const int64_t work = (tiles + kEwBlock / 32 - 1) / (kEwBlock / 32);
#define CTB_RM(M, B)                                                                             \
    {                                                                                            \
        auto k = &ew_rows_mid<Fn, O, I0, I1, I2, NIN, M, kRowsMidUnroll, B>;                     \
        launch_dependent(k, wave_grid(k, work), kEwBlock, 0, st, a, fn);                                       \
    }
        switch (inner_mask(a, NIN)) {
        case 0: CTB_RM(0, (rows_min_blocks<O, I0, I1, I2, NIN, 0>())) break;
        case 1: CTB_RM(1, (rows_min_blocks<O, I0, I1, I2, NIN, 1>())) break;
        case 2:
            if constexpr (NIN > 1) {
                if constexpr (RowPrep<Fn>::kActive) CTB_RM(2, kRowDivMinBlocks)
                else CTB_RM(2, (rows_min_blocks<O, I0, I1, I2, NIN, 2>()))
                break;
            }
            [[fallthrough]];
        default: CTB_RM(-1, 2) break;
        }
#undef CTB_RM
        break;
    }
    case EwPath::RowsShort: {
        const int64_t nvec = a.rows * a.vpr;
        const int64_t work = (nvec + kEwBlock * kEwUnroll - 1) / (kEwBlock * kEwUnroll);
#define CTB_RS(M, B)                                                     \
    {                                                                    \
        auto k = &ew_rows_short<Fn, O, I0, I1, I2, NIN, M, B>;           \
        launch_dependent(k, wave_grid(k, work), kEwBlock, 0, st, a, fn);               \
    }
        switch (inner_mask(a, NIN)) {
        case 0: CTB_RS(0, (rows_min_blocks<O, I0, I1, I2, NIN, 0>())) break;
        case 1: CTB_RS(1, (rows_min_blocks<O, I0, I1, I2, NIN, 1>())) break;
        case 2:
            if constexpr (NIN > 1) {
                if constexpr (RowPrep<Fn>::kActive) CTB_RS(2, kRowDivMinBlocks)
                else CTB_RS(2, (rows_min_blocks<O, I0, I1, I2, NIN, 2>()))
                break;
            }
            [[fallthrough]];
        default: CTB_RS(-1, 2) break;
        }
#undef CTB_RS
        break;
    }
    case EwPath::Tiled: {
        if constexpr (NIN == 2) {
            const int64_t L = a.shape[a.rank - 1];
            const int64_t P = a.shape[a.pdim];
            const int64_t total = (a.n / (L * P)) * static_cast<int64_t>(a.aux.d) * static_cast<int64_t>(a.aux2.d);
            // 128-wide tiles along l (512 threads) for 4-byte types (8-byte ones already move
            // 512-byte runs with 64-wide tiles); tiles along l recounted for them
            constexpr bool kWideL = sizeof(I0) == 4 && sizeof(I1) == 4 && sizeof(O) == 4;
            bool wide_done = false;
            if constexpr (kWideL) {
              if (a.tiled_vec && L >= 2 * kTile) {
                EwArgs aw = a;
                aw.aux = FastDiv(static_cast<uint64_t>((L + 2 * kTile - 1) / (2 * kTile)));
                const int64_t tw = (a.n / (L * P)) * static_cast<int64_t>(aw.aux.d) * static_cast<int64_t>(aw.aux2.d);
                auto launch = [&](auto k) {
                    const int64_t slots = static_cast<int64_t>(sm_count()) *
                                          resident_ctas(reinterpret_cast<const void*>(k), 2 * kEwBlock);
                    const int64_t g = tw < slots ? tw : slots;
                    launch_dependent(k, static_cast<unsigned>(g < 1 ? 1 : g), 2 * kEwBlock, 0, st, aw, fn);
                };
                if (a.xop == 1) launch(&ew_tiled4<Fn, O, I0, I1, 1, 2 * kTile>);
                else launch(&ew_tiled4<Fn, O, I0, I1, 2, 2 * kTile>);
                wide_done = true;
              }
            }
            if (wide_done) {
            } else if (a.tiled_vec) {
                if (a.xop == 1) {
                    auto k = &ew_tiled4<Fn, O, I0, I1, 1>;
                    launch_dependent(k, wave_grid(k, total), kEwBlock, 0, st, a, fn);
                } else {
                    auto k = &ew_tiled4<Fn, O, I0, I1, 2>;
                    launch_dependent(k, wave_grid(k, total), kEwBlock, 0, st, a, fn);
                }
            } else if (a.xop == 1) {
                launch_dependent(ew_tiled<Fn, O, I0, I1, 1>, grid_for(total, 16), kEwBlock, 0, st, a, fn);
            } else {
                launch_dependent(ew_tiled<Fn, O, I0, I1, 2>, grid_for(total, 16), kEwBlock, 0, st, a, fn);
            }
            break;
        }
        [[fallthrough]];
    }
    case EwPath::General: {
        launch_dependent(ew_general<Fn, O, I0, I1, I2, NIN>, grid_for((a.n + kEwBlock - 1) / kEwBlock, 16), kEwBlock, 0, st, a, fn);
        break;
    }
    }
    count_launch();
    return check_launch("elementwise");
}

// ------------------------------------------------------------------------------------------------
// op2(op1(a, b) rounded to M, c) rounded to O.
template <int OP1, int OP2, class M, class O> struct FnChain {
    static constexpr bool kWideRows = OP1 != CTB_DIV && OP2 != CTB_DIV;
    template <class A, class B, class C> __device__ __forceinline__ O operator()(A a, B b, C c) const {
        const M m = BinOp<OP1>::template apply<M>(cvt<M>(a), cvt<M>(b));
        return BinOp<OP2>::template apply<O>(cvt<O>(m), cvt<O>(c));
    }
};

}  // namespace ctb
