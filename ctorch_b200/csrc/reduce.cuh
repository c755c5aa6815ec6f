// reduce.cuh — sm_100a reduction kernels (sum / mean / prod / max / min, with or without indices).
//
// A reducer R supplies State, init(), fold(state, value, position), combine(state, state) and
// write(). Kernels (chosen by plan_reduction / finish_reduction_plan in plan.cu):
//   red_inner_cta   reduced range contiguous (row reductions, whole-tensor sums): one CTA per
//                   (row, split), 16-byte loads four deep, warp-shuffle then shared-memory tree
//   red_inner_warp  same for short rows: one warp per row
//   red_outer       reduced dim strided, kept dim contiguous (column reductions): each warp walks
//                   rows of a 32*V-column strip, warps combine through shared memory
//   red_runs_cta    other layouts whose innermost reduced dim is contiguous: 16-byte packs along
//                   the runs, each pack's run decoded once
//   red_general_*   any other layout: per-element coordinate decode
//   red_finalize    deterministic fixed-order combine of split partials (the second pass);
//                   red_finalize_cta for few outputs with many partials (a CTA-wide fixed tree)
// Replaces ctorch's one-thread-per-output axis kernels and whole-tensor two-pass kernels
// (src/ops/reduction_ops_cuda.cu:92-350).
//
// Determinism and parity: every combine order is fixed by the launch shape, which depends only
// on the problem size and the SM count, so results are run-to-run identical. Integer sums and
// products accumulate in uint64 (two's-complement wrap, identical to any order); float sums and
// products accumulate in double; max/min carry the element's position so ties resolve to the
// first occurrence and NaN to the first NaN, exactly as the sequential CPU fold
// (src/ops/reduction_functors.h:55-110, src/ops/reduction_ops_cpu.cpp:236-297).
#pragma once

#include <limits>
#include <mutex>

#include "async_copy.cuh"
#include "common.cuh"
#include "plan.cuh"

namespace ctb {

constexpr int kRedBlock = 256;
constexpr int kOuterBlock = 128;  // column strips: 4 warps, so twice the resident CTAs to spread over

// Packs each thread keeps in flight (R::kUnroll): sums and products of 4-byte elements keep 8
// (a warp has 4 KiB of loads outstanding per step); max/min states carry a position as well, so
// they keep 4 to stay at 4 resident CTAs per SM.
template <class R> constexpr int red_unroll() { return R::kUnroll; }

// ------------------------------------------------------------------------------------------------
// shuffles

template <class T> __device__ __forceinline__ T shfl_xor(T v, int m) {
    if constexpr (std::is_same_v<T, uint8_t>) {
        return static_cast<uint8_t>(__shfl_xor_sync(0xffffffffu, static_cast<int>(v), m));
    } else if constexpr (std::is_same_v<T, int64_t>) {
        return static_cast<int64_t>(__shfl_xor_sync(0xffffffffu, static_cast<long long>(v), m));
    } else if constexpr (std::is_same_v<T, uint64_t>) {
        return static_cast<uint64_t>(
            __shfl_xor_sync(0xffffffffu, static_cast<unsigned long long>(v), m));
    } else {
        return __shfl_xor_sync(0xffffffffu, v, m);
    }
}

// ------------------------------------------------------------------------------------------------
// reducers

// Sum / product with a widening accumulator: double for float inputs, uint64 (wrapping) for
// integer and bool inputs (src/ops/reduction_ops_cpu.cpp:98-152).
template <class T, bool IsProd> struct RAccum {
    using In = T;
    using State = std::conditional_t<is_float_v<T>, double, uint64_t>;
    using Out = std::conditional_t<is_float_v<T>, T, int64_t>;
    static constexpr int kUnroll = sizeof(T) <= 4 ? 8 : 4;
    __device__ __forceinline__ static State init() { return IsProd ? State(1) : State(0); }
    __device__ __forceinline__ static State conv(T v) {
        if constexpr (is_float_v<T>) return static_cast<double>(v);
        else if constexpr (std::is_same_v<T, uint8_t>) return static_cast<uint64_t>(v);
        else return static_cast<uint64_t>(static_cast<int64_t>(v));
    }
    __device__ __forceinline__ static void combine(State& a, State b) {
        if constexpr (is_float_v<T>) a = IsProd ? __dmul_rn(a, b) : __dadd_rn(a, b);
        else a = IsProd ? a * b : a + b;
    }
    __device__ __forceinline__ static void fold(State& s, T v, int64_t) { combine(s, conv(v)); }
    // Per-thread state over a chunk of at most 2^31 - 1 positions (see RMinMax::Local).
    using Local = State;
    __device__ __forceinline__ static Local local_init() { return init(); }
    __device__ __forceinline__ static void fold_local(Local& s, T v, int32_t) { combine(s, conv(v)); }
    __device__ __forceinline__ static State widen(const Local& s, int64_t) { return s; }
    __device__ __forceinline__ static State shfl(State s, int m) { return shfl_xor(s, m); }
    __device__ __forceinline__ static void write(const RedArgs& p, const State& s, int64_t o1, int64_t) {
        if constexpr (is_float_v<T>) static_cast<T*>(p.out)[o1] = static_cast<T>(s);
        else static_cast<int64_t*>(p.out)[o1] = static_cast<int64_t>(s);
    }
};

// mean = T(sum) then *= T(1)/T(N); NaN (ctorch's quiet_NaN bits) when N == 0
// (src/ops/reduction_ops_cpu.cpp:160-175).
template <class T> struct RMean : RAccum<T, false> {
    using Base = RAccum<T, false>;
    using State = typename Base::State;
    __device__ __forceinline__ static void write(const RedArgs& p, const State& s, int64_t o1, int64_t) {
        T o;
        if (p.red == 0) {
            if constexpr (std::is_same_v<T, float>) o = __int_as_float(0x7fc00000);
            else o = __longlong_as_double(0x7ff8000000000000LL);
        } else {
            o = static_cast<T>(s);
            if constexpr (std::is_same_v<T, float>)
                o = __fmul_rn(o, __fdiv_rn(1.0f, static_cast<float>(p.red)));
            else
                o = __dmul_rn(o, __ddiv_rn(1.0, static_cast<double>(p.red)));
        }
        static_cast<T*>(p.out)[o1] = o;
    }
};

// Sum of a float shard into a double partial (multi-GPU whole-tensor sum).
template <class T> struct RSumPartial : RAccum<T, false> {
    using State = typename RAccum<T, false>::State;
    __device__ __forceinline__ static void write(const RedArgs& p, const State& s, int64_t o1, int64_t) {
        static_cast<double*>(p.out)[o1] = s;
    }
};

template <class T> struct MMState {
    T v;
    int64_t i;
};

// max / min carrying the position: NaN beats numbers (first NaN wins), then the larger (smaller)
// value, then the smaller position. Equivalent to ctorch's sequential strict-compare fold.
template <class T, bool IsMax, bool Indexed> struct RMinMax {
    using In = T;
    using State = MMState<T>;
    static constexpr int kUnroll = 4;
    __device__ __forceinline__ static T ident() {
        if constexpr (is_float_v<T>)
            return IsMax ? -std::numeric_limits<T>::infinity() : std::numeric_limits<T>::infinity();
        else
            return IsMax ? std::numeric_limits<T>::lowest() : std::numeric_limits<T>::max();
    }
    __device__ __forceinline__ static State init() {
        return State{ident(), std::numeric_limits<int64_t>::max()};
    }
    __device__ __forceinline__ static bool better(const State& a, T bv, int64_t bi) {
        if constexpr (is_float_v<T>) {
            const bool an = a.v != a.v, bn = bv != bv;
            if (an | bn) return an ? (bn && bi < a.i) : true;
        }
        if (IsMax ? (bv > a.v) : (bv < a.v)) return true;
        return bv == a.v && bi < a.i;
    }
    // Every kernel folds a thread's elements in increasing position order, so a strict compare
    // keeps the first occurrence and a NaN, once adopted, is kept (the sequential CPU rule). A
    // state that has only met the identity value (+-inf, or the integer limit) keeps the "empty"
    // position INT64_MAX; `combine` applies the full rule, and `write` maps an all-identity
    // slice to position 0, its first element.
    // take v when the state is not NaN and v is NaN or strictly better: for floats that is
    // "s.v is a number and not (v <= s.v)" (not (v >= s.v) for min), two compares.
    __device__ __forceinline__ static bool takes(T sv, T v) {
        if constexpr (is_float_v<T>) return (sv == sv) && !(IsMax ? v <= sv : v >= sv);
        else return IsMax ? v > sv : v < sv;
    }
    __device__ __forceinline__ static void fold(State& s, T v, int64_t j) {
        if (takes(s.v, v)) {
            s.v = v;
            s.i = j;
        }
    }
    // A thread's state over one chunk of positions [base, base + 2^31 - 1): the position is kept
    // as a 32-bit offset from base (one register and one select less per element); widen()
    // turns it back into the 64-bit state, keeping "empty" as INT64_MAX.
    struct Local {
        T v;
        int32_t i;
    };
    __device__ __forceinline__ static Local local_init() {
        return Local{ident(), std::numeric_limits<int32_t>::max()};
    }
    __device__ __forceinline__ static void fold_local(Local& s, T v, int32_t j) {
        if (takes(s.v, v)) {
            s.v = v;
            s.i = j;
        }
    }
    __device__ __forceinline__ static State widen(const Local& s, int64_t base) {
        return State{s.v, s.i == std::numeric_limits<int32_t>::max() ? std::numeric_limits<int64_t>::max()
                                                                      : base + s.i};
    }
    __device__ __forceinline__ static void combine(State& a, const State& b) {
        if (better(a, b.v, b.i)) a = b;
    }
    __device__ __forceinline__ static State shfl(const State& s, int m) {
        return State{shfl_xor(s.v, m), shfl_xor(s.i, m)};
    }
    __device__ __forceinline__ static void write(const RedArgs& p, const State& s, int64_t o1, int64_t o2) {
        if (p.out) static_cast<T*>(p.out)[o1] = s.v;
        if constexpr (Indexed)
            static_cast<int64_t*>(p.out2)[o2] = s.i == std::numeric_limits<int64_t>::max() ? 0 : s.i;
    }
};

// ------------------------------------------------------------------------------------------------
// helpers

template <class R> __device__ __forceinline__ typename R::State warp_reduce(typename R::State s) {
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) R::combine(s, R::shfl(s, m));
    return s;
}

// Result valid in thread 0. `smem` holds one State per warp.
template <class R> __device__ __forceinline__ typename R::State block_reduce(typename R::State s,
                                                                             typename R::State* smem) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nwarps = blockDim.x >> 5;
    s = warp_reduce<R>(s);
    if (lane == 0) smem[warp] = s;
    __syncthreads();
    if (warp == 0) {
        s = lane < nwarps ? smem[lane] : R::init();
        s = warp_reduce<R>(s);
    }
    __syncthreads();
    return s;
}

// Offsets of kept index k: input, first output, second output.
__device__ __forceinline__ void red_decode_kept(const RedArgs& p, uint64_t k, int64_t& in_off,
                                                int64_t& o1, int64_t& o2) {
    in_off = o1 = o2 = 0;
    for (int d = p.rank_k - 1; d >= 0; --d) {
        uint64_t q, c;
        p.div_k[d].divmod(k, q, c);
        in_off += static_cast<int64_t>(c) * p.stride_k[d];
        o1 += static_cast<int64_t>(c) * p.stride_o[d];
        o2 += static_cast<int64_t>(c) * p.stride_o2[d];
        k = q;
    }
}

__device__ __forceinline__ int64_t red_decode_red(const RedArgs& p, uint64_t j) {
    int64_t off = 0;
    for (int d = p.rank_r - 1; d >= 0; --d) {
        uint64_t q, c;
        p.div_r[d].divmod(j, q, c);
        off += static_cast<int64_t>(c) * p.stride_r[d];
        j = q;
    }
    return off;
}

// Offset of run r of the reduced subspace whose innermost dim (rank_r - 1) is contiguous: r
// decoded over the outer reduced dims only, the outermost without a divide (its coordinate is
// what is left). Two reduced dims cost one multiply.
__device__ __forceinline__ int64_t red_decode_run(const RedArgs& p, uint64_t r) {
    int64_t off = 0;
    for (int d = p.rank_r - 2; d > 0; --d) {
        uint64_t q, c;
        p.div_r[d].divmod(r, q, c);
        off += static_cast<int64_t>(c) * p.stride_r[d];
        r = q;
    }
    return off + static_cast<int64_t>(r) * p.stride_r[0];
}

// Folds row[j] for j in [j0, j1) into s, elements spread over nthr threads: scalar head up to
// the first 16-byte boundary, 16-byte packs R::kUnroll deep, scalar tail.
template <class R> __device__ __forceinline__ void fold_contig(const typename R::In* row, int64_t j0,
                                                               int64_t j1, typename R::State& s,
                                                               int tid, int nthr) {
    using T = typename R::In;
    constexpr int V = 16 / sizeof(T);
    constexpr int U = red_unroll<R>();
    if (j1 <= j0) return;
    const uintptr_t addr = reinterpret_cast<uintptr_t>(row + j0);
    const int64_t head = static_cast<int64_t>(((16u - (addr & 15u)) & 15u) / sizeof(T));
    const int64_t jh = j0 + head < j1 ? j0 + head : j1;
    for (int64_t j = j0 + tid; j < jh; j += nthr) R::fold(s, row[j], j);
    const int64_t nv = (j1 - jh) / V;
    const T* body = row + jh;
    for (int64_t v = tid; v < nv; v += static_cast<int64_t>(nthr) * U) {
        Pack<T, V> x[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t w = v + static_cast<int64_t>(u) * nthr;
            if (w < nv) x[u] = load_pack<T, V>(body + w * V);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t w = v + static_cast<int64_t>(u) * nthr;
            if (w < nv) {
#pragma unroll
                for (int e = 0; e < V; ++e) R::fold(s, x[u].v[e], jh + w * V + e);
            }
        }
    }
    for (int64_t j = jh + nv * V + tid; j < j1; j += nthr) R::fold(s, row[j], j);
}

// ------------------------------------------------------------------------------------------------
// kernels

template <class R> __global__ void __launch_bounds__(kRedBlock) red_inner_cta(RedArgs p) {
    dependent_wait();  // the previous kernel in the stream has completed and its writes are visible
    allow_dependents();  // one-wave grid: the next kernel (a second pass or the next op) may launch now
    using T = typename R::In;
    using S = typename R::State;
    __shared__ S smem[32];
    const int64_t total = p.kept * p.split;
    for (int64_t t = blockIdx.x; t < total; t += gridDim.x) {
        uint64_t row, sp;
        p.aux.divmod(static_cast<uint64_t>(t), row, sp);
        int64_t in_off, o1, o2;
        red_decode_kept(p, row, in_off, o1, o2);
        const T* base = static_cast<const T*>(p.in) + in_off;
        const int64_t j0 = static_cast<int64_t>(sp) * p.chunk;
        const int64_t j1 = j0 + p.chunk < p.K ? j0 + p.chunk : p.K;
        S st = R::init();
        fold_contig<R>(base, j0, j1, st, threadIdx.x, blockDim.x);
        st = block_reduce<R>(st, smem);
        if (threadIdx.x == 0) {
            if (p.split == 1) R::write(p, st, o1, o2);
            else static_cast<S*>(p.scratch)[t] = st;
        }
    }
}

template <class R> __global__ void __launch_bounds__(kRedBlock) red_inner_warp(RedArgs p) {
    dependent_wait();  // the previous kernel in the stream has completed and its writes are visible
    allow_dependents();  // one-wave grid: the next kernel (a second pass or the next op) may launch now
    using T = typename R::In;
    using S = typename R::State;
    const int lane = threadIdx.x & 31;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    for (int64_t row = warp; row < p.kept; row += nwarps) {
        int64_t in_off, o1, o2;
        red_decode_kept(p, static_cast<uint64_t>(row), in_off, o1, o2);
        S st = R::init();
        fold_contig<R>(static_cast<const T*>(p.in) + in_off, 0, p.K, st, lane, 32);
        st = warp_reduce<R>(st);
        if (lane == 0) R::write(p, st, o1, o2);
    }
}

// Rows shared by a group of G warps (G = 2 or 4) of one CTA, for long rows that are too few to
// keep every warp busy one row each to the end (8192 rows of 32 KiB over ~4700 warps leave the
// second round of rows 70% full). The G warps fold interleaved packs of the row, then the
// group's warp results are combined in warp order through shared memory (double-buffered by row
// parity, one named barrier per row for the group's warps only).
template <class R, int G> __global__ void __launch_bounds__(kRedBlock) red_inner_group(RedArgs p) {
    dependent_wait();  // the previous kernel in the stream has completed and its writes are visible
    allow_dependents();  // one-wave grid: the next kernel (a second pass or the next op) may launch now
    using T = typename R::In;
    using S = typename R::State;
    constexpr int kGroups = kRedBlock / (32 * G);
    __shared__ S part[2][kGroups][G];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int gib = wib / G, wig = wib % G;
    const int64_t ngroups = static_cast<int64_t>(gridDim.x) * kGroups;
    int parity = 0;
    for (int64_t row = static_cast<int64_t>(blockIdx.x) * kGroups + gib; row < p.kept; row += ngroups) {
        int64_t in_off, o1, o2;
        red_decode_kept(p, static_cast<uint64_t>(row), in_off, o1, o2);
        S st = R::init();
        fold_contig<R>(static_cast<const T*>(p.in) + in_off, 0, p.K, st, wig * 32 + lane, 32 * G);
        st = warp_reduce<R>(st);
        if (lane == 0) part[parity][gib][wig] = st;
        asm volatile("bar.sync %0, %1;" ::"r"(1 + gib), "r"(32 * G) : "memory");
        if (wig == 0 && lane == 0) {
            S acc = part[parity][gib][0];
#pragma unroll
            for (int w = 1; w < G; ++w) R::combine(acc, part[parity][gib][w]);
            R::write(p, acc, o1, o2);
        }
        parity ^= 1;
    }
}

// Column strips: kept inner dim N contiguous, reduced dim K with stride strideK, batch dims in
// front. CTA = 8 warps; warp w folds rows k0+w, k0+w+8, ... of a 32*V-column strip.
template <class R, int V> __global__ void __launch_bounds__(kOuterBlock) red_outer(RedArgs p) {
    dependent_wait();  // the previous kernel in the stream has completed and its writes are visible
    allow_dependents();  // one-wave grid: the next kernel (a second pass or the next op) may launch now
    using T = typename R::In;
    using S = typename R::State;
    constexpr int W = kOuterBlock / 32;
    // rows in flight per warp: a column strip is one 16-byte pack per lane per row, so keep 8 rows
    // of 4-byte elements (4 KiB per warp) outstanding
    constexpr int U = sizeof(T) <= 4 ? 8 : 4;
    __shared__ S smem[W - 1][32 * V];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t tiles_n = static_cast<int64_t>(p.aux.d);
    const int64_t total = (p.kept / p.N) * tiles_n * p.split;
    for (int64_t t = blockIdx.x; t < total; t += gridDim.x) {
        uint64_t rest, sp, b, tn;
        p.aux2.divmod(static_cast<uint64_t>(t), rest, sp);
        p.aux.divmod(rest, b, tn);
        int64_t in_off = 0, o1 = 0, o2 = 0;
        {
            uint64_t bb = b;
            for (int d = p.rank_k - 2; d >= 0; --d) {
                uint64_t q, c;
                p.div_k[d].divmod(bb, q, c);
                in_off += static_cast<int64_t>(c) * p.stride_k[d];
                o1 += static_cast<int64_t>(c) * p.stride_o[d];
                o2 += static_cast<int64_t>(c) * p.stride_o2[d];
                bb = q;
            }
        }
        const int64_t col0 = static_cast<int64_t>(tn) * (32 * V) + lane * V;
        const int64_t k0 = static_cast<int64_t>(sp) * p.chunk;
        const int64_t k1 = k0 + p.chunk < p.K ? k0 + p.chunk : p.K;
        // positions are folded as 32-bit offsets from k0 (the plan keeps chunks below 2^31)
        typename R::Local lst[V];
#pragma unroll
        for (int e = 0; e < V; ++e) lst[e] = R::local_init();
        const T* base = static_cast<const T*>(p.in) + in_off + col0;
        if (col0 + V <= p.N) {
            for (int64_t k = k0 + warp; k < k1; k += W * U) {
                Pack<T, V> x[U];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int64_t kk = k + u * W;
                    if (kk < k1) x[u] = load_pack<T, V>(base + kk * p.strideK);
                }
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int64_t kk = k + u * W;
                    if (kk < k1) {
                        const int32_t j = static_cast<int32_t>(kk - k0);
#pragma unroll
                        for (int e = 0; e < V; ++e) R::fold_local(lst[e], x[u].v[e], j);
                    }
                }
            }
        } else {
            for (int64_t k = k0 + warp; k < k1; k += W) {
                const int32_t j = static_cast<int32_t>(k - k0);
#pragma unroll
                for (int e = 0; e < V; ++e)
                    if (col0 + e < p.N) R::fold_local(lst[e], base[k * p.strideK + e], j);
            }
        }
        S st[V];
#pragma unroll
        for (int e = 0; e < V; ++e) st[e] = R::widen(lst[e], k0);
        if (warp > 0) {
#pragma unroll
            for (int e = 0; e < V; ++e) smem[warp - 1][lane * V + e] = st[e];
        }
        __syncthreads();
        if (warp == 0) {
#pragma unroll
            for (int e = 0; e < V; ++e) {
                for (int w = 0; w < W - 1; ++w) R::combine(st[e], smem[w][lane * V + e]);
                const int64_t col = col0 + e;
                if (col < p.N) {
                    if (p.split == 1) {
                        R::write(p, st[e], o1 + col, o2 + col);
                    } else {
                        const int64_t k = static_cast<int64_t>(b) * p.N + col;
                        static_cast<S*>(p.scratch)[k * p.split + static_cast<int64_t>(sp)] = st[e];
                    }
                }
            }
        }
        __syncthreads();
    }
}

// ------------------------------------------------------------------------------------------------
// Column reductions through a shared-memory stage ring filled by bulk asynchronous copies
// (async_copy.cuh). Warp 4 is the producer: for each stage it copies 8 rows of a column tile (2 KiB
// of each row, one bulk copy per row, issued by one lane each) into shared memory. Warps 0-3 are
// consumers: thread t owns one 16-byte pack of the tile's columns (4 float columns) and folds them
// down the stage in row order, one independent chain per column, so the fold order per output is
// the row order, as in ctorch's sequential fold. The CTA's loads are in flight in the copy engine,
// not in registers: 6 stages of 16 KiB keep 96 KiB per CTA moving.
//
// Work split (stream-K): the column tiles x rows form one sequence of row-steps; CTA c takes an
// equal contiguous share of it (RedArgs::sk_q, sk_r). A tile a CTA covers whole is written
// directly; a tile s shared by several CTAs gets one partial state per column from each CTA c
// that touches it (scratch row c + s), combined in CTA order by red_cols_finalize.

constexpr int kColsStages = 6;
template <class T> constexpr int cols_tile() { return kColsRowBytes / static_cast<int>(sizeof(T)); }
constexpr size_t cols_smem_bytes() {
    return static_cast<size_t>(kColsStages) * kColsRows * kColsRowBytes + 2 * kColsStages * sizeof(uint64_t);
}

// Tile s of the bulk column kernel: input offset of its first column, output offsets of its
// batch row, and its first column.
template <class T>
__device__ __forceinline__ void cols_tile_at(const RedArgs& p, uint64_t s, int64_t& in_off, int64_t& o1,
                                             int64_t& o2, int64_t& col0) {
    uint64_t b, tn;
    p.aux.divmod(s, b, tn);
    in_off = o1 = o2 = 0;
    for (int d = p.rank_k - 2; d >= 0; --d) {
        uint64_t q, c;
        p.div_k[d].divmod(b, q, c);
        in_off += static_cast<int64_t>(c) * p.stride_k[d];
        o1 += static_cast<int64_t>(c) * p.stride_o[d];
        o2 += static_cast<int64_t>(c) * p.stride_o2[d];
        b = q;
    }
    col0 = static_cast<int64_t>(tn) * cols_tile<T>();
}

__device__ __forceinline__ int64_t cols_start(const RedArgs& p, int64_t c) {
    return c * p.sk_q + (c < p.sk_r ? c : p.sk_r);
}

template <class R> __global__ void __launch_bounds__(kColsThreads, 1) red_cols_bulk(RedArgs p) {
    dependent_wait();  // the previous kernel in the stream has completed and its writes are visible
    // The consumers let the dependent second pass (red_cols_finalize) launch only once they have
    // folded their last stage: finalize CTAs resident beside this kernel from its start slowed
    // its stream, while a trigger at the end hides the finalize's launch behind this kernel's
    // tail (argmax over dim 0 of [8192, 8192] float32 on B200: 52.2 -> 49.6 us for both passes).
    using T = typename R::In;
    using S = typename R::State;
    constexpr int NS = kColsStages;
    constexpr int VE = 16 / static_cast<int>(sizeof(T));  // columns per consumer thread
    constexpr int TW = cols_tile<T>();                      // columns per tile
    constexpr int kStage = kColsRows * TW;                  // elements per stage
    constexpr int kConsumerWarps = kColsConsumers / 32;
    extern __shared__ __align__(128) unsigned char cols_smem[];
    T* stages = reinterpret_cast<T*>(cols_smem);
    uint64_t* full = reinterpret_cast<uint64_t*>(cols_smem + static_cast<size_t>(NS) * kStage * sizeof(T));
    uint64_t* empty = full + NS;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < NS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kConsumerWarps);
        }
        mbar_fence_init();
    }
    __syncthreads();

    const int64_t c = blockIdx.x;
    const int64_t start = cols_start(p, c);
    const int64_t end = cols_start(p, c + 1);
    if (warp == kConsumerWarps) {
        // ---- producer
        uint32_t g = 0;
        bool ok = true;
        for (int64_t pos = start; pos < end && ok;) {
            uint64_t s, ka;
            p.aux2.divmod(static_cast<uint64_t>(pos), s, ka);
            const int64_t kb = min(p.K, static_cast<int64_t>(ka) + (end - pos));
            int64_t in_off, o1, o2, col0;
            cols_tile_at<T>(p, s, in_off, o1, o2, col0);
            const T* src = static_cast<const T*>(p.in) + in_off + col0;
            const int64_t ncols = min(static_cast<int64_t>(TW), p.N - col0);
            const uint32_t vb = static_cast<uint32_t>(ncols * static_cast<int64_t>(sizeof(T)));
            for (int64_t k = static_cast<int64_t>(ka); k < kb; k += kColsRows, ++g) {
                const int slot = static_cast<int>(g % NS);
                const bool w = mbar_wait(&empty[slot], ((g / NS) & 1u) ^ 1u);
                if (!__all_sync(0xffffffffu, w)) {
                    ok = false;
                    break;
                }
                const int rows = static_cast<int>(min(static_cast<int64_t>(kColsRows), kb - k));
                if (lane == 0) mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(rows) * vb);
                __syncwarp();
                if (lane < rows)
                    bulk_load(stages + slot * kStage + lane * TW, src + (k + lane) * p.strideK, vb, &full[slot]);
            }
            pos += kb - static_cast<int64_t>(ka);
        }
        if (!ok && lane == 0) {
            note_timeout(p.timeouts);
            // let the copies already issued land before the CTA's shared memory goes away
            for (uint32_t i = g > static_cast<uint32_t>(NS) ? g - NS : 0u; i < g; ++i)
                mbar_wait(&full[i % NS], (i / NS) & 1u);
        }
        return;
    }

    // ---- consumers: thread t folds columns [t*VE, t*VE + VE) of the tile
    const int t = threadIdx.x;
    uint32_t g = 0;
    for (int64_t pos = start; pos < end;) {
        uint64_t s, ka;
        p.aux2.divmod(static_cast<uint64_t>(pos), s, ka);
        const int64_t kb = min(p.K, static_cast<int64_t>(ka) + (end - pos));
        int64_t in_off, o1, o2, col0;
        cols_tile_at<T>(p, s, in_off, o1, o2, col0);
        const int64_t col = col0 + static_cast<int64_t>(t) * VE;
        const bool active = col < p.N;  // N is a whole number of packs, so a pack is all in or out
        typename R::Local st[VE];
#pragma unroll
        for (int e = 0; e < VE; ++e) st[e] = R::local_init();
        for (int64_t k = static_cast<int64_t>(ka); k < kb; k += kColsRows, ++g) {
            const int slot = static_cast<int>(g % NS);
            const bool w = mbar_wait(&full[slot], (g / NS) & 1u);
            if (!__all_sync(0xffffffffu, w)) {
                if (lane == 0) note_timeout(p.timeouts);
                return;
            }
            const int rows = static_cast<int>(min(static_cast<int64_t>(kColsRows), kb - k));
            const T* sb = stages + slot * kStage + t * VE;
            const int32_t j0 = static_cast<int32_t>(k - static_cast<int64_t>(ka));
            if (active) {
                if (rows == kColsRows) {
                    Pack<T, VE> x[kColsRows];
#pragma unroll
                    for (int j = 0; j < kColsRows; ++j) x[j] = *reinterpret_cast<const Pack<T, VE>*>(sb + j * TW);
#pragma unroll
                    for (int j = 0; j < kColsRows; ++j)
#pragma unroll
                        for (int e = 0; e < VE; ++e) R::fold_local(st[e], x[j].v[e], j0 + j);
                } else {
                    for (int j = 0; j < rows; ++j) {
                        const Pack<T, VE> x = *reinterpret_cast<const Pack<T, VE>*>(sb + j * TW);
#pragma unroll
                        for (int e = 0; e < VE; ++e) R::fold_local(st[e], x.v[e], j0 + j);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
        if (pos + (kb - static_cast<int64_t>(ka)) >= end) allow_dependents();
        if (active) {
            const bool whole = ka == 0 && kb == p.K;
            S* part = static_cast<S*>(p.scratch) + (c + static_cast<int64_t>(s)) * TW + t * VE;
#pragma unroll
            for (int e = 0; e < VE; ++e) {
                const S v = R::widen(st[e], static_cast<int64_t>(ka));
                if (whole) R::write(p, v, o1 + col + e, o2 + col + e);
                else part[e] = v;
            }
        }
        pos += kb - static_cast<int64_t>(ka);
    }
}

// Second pass of the bulk column kernel: for every column of a tile shared by several CTAs,
// combine their partial states in CTA order (that is, row order) and write the result. A block
// takes 32 consecutive outputs (one per lane, so partial loads are coalesced) and splits each one's
// CTA range into 8 consecutive groups, one per warp; warp 0 then combines the 8 group results in
// group order. The combine order is fixed by the plan, so results are run-to-run identical.
constexpr int kColsFixGroups = 8;
template <class R> __global__ void __launch_bounds__(32 * kColsFixGroups) red_cols_finalize(RedArgs p) {
    dependent_wait();  // the first pass has completed and its partials are visible
    allow_dependents();  // small kernel: the next one in the stream may launch during it
    using T = typename R::In;
    using S = typename R::State;
    constexpr int TW = cols_tile<T>();
    __shared__ S red[kColsFixGroups][32];
    const int lane = threadIdx.x & 31, grp = threadIdx.x >> 5;
    const S* part = static_cast<const S*>(p.scratch);
    const int64_t tiles_n = static_cast<int64_t>(p.aux.d);
    const int64_t big = p.sk_r * (p.sk_q + 1);  // row-steps owned by the CTAs with one extra
    for (int64_t k0 = static_cast<int64_t>(blockIdx.x) * 32; k0 < p.kept; k0 += static_cast<int64_t>(gridDim.x) * 32) {
        const int64_t k = k0 + lane;
        bool shared_tile = false;
        S st = R::init();
        if (k < p.kept) {
            const int64_t b = k / p.N, col = k - b * p.N;
            const int64_t s = b * tiles_n + col / TW;
            const int64_t first = s * p.K, last = first + p.K - 1;
            const int64_t c_lo = first < big ? first / (p.sk_q + 1) : p.sk_r + (first - big) / p.sk_q;
            const int64_t c_hi = last < big ? last / (p.sk_q + 1) : p.sk_r + (last - big) / p.sk_q;
            shared_tile = c_lo != c_hi;  // else one CTA covered the whole tile and wrote it
            if (shared_tile) {
                const int64_t n = c_hi - c_lo + 1;
                const int64_t per = (n + kColsFixGroups - 1) / kColsFixGroups;
                const int64_t ca = c_lo + grp * per;
                const int64_t cb = min(c_hi + 1, ca + per);
                const S* col_parts = part + s * TW + col % TW;
                int64_t cc = ca;
                for (; cc + 4 <= cb; cc += 4) {
                    S v[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) v[u] = col_parts[(cc + u) * TW];
#pragma unroll
                    for (int u = 0; u < 4; ++u) R::combine(st, v[u]);
                }
                for (; cc < cb; ++cc) R::combine(st, col_parts[cc * TW]);
            }
        }
        red[grp][lane] = st;
        __syncthreads();
        if (grp == 0 && shared_tile) {
            S r = red[0][lane];
#pragma unroll
            for (int g2 = 1; g2 < kColsFixGroups; ++g2) R::combine(r, red[g2][lane]);
            int64_t in_off, o1, o2;
            red_decode_kept(p, static_cast<uint64_t>(k), in_off, o1, o2);
            R::write(p, r, o1, o2);
        }
        __syncthreads();
    }
}

// ------------------------------------------------------------------------------------------------
// Column reductions by strips of whole columns (4- and 8-byte types). A unit is one strip of one
// batch row: up to PK 16-byte packs of columns over all K rows. CTA c takes units c, c + grid, ...
// and folds each one completely, so every output is written once, by one CTA, with no partial
// states and no second pass.
//
// Warp 8 is the producer: each stage is one tensor copy of RPS = Q * kStripRows rows of the strip
// (the box of the kernel's tensor map), landing as RPS rows of PK packs back to back. The 256
// consumer threads form Q = 256 / PK row groups; thread (q, j) owns pack j of the strip and folds
// rows q, q + Q, q + 2Q, ... of each stage, kStripRows of them, in increasing row order. So the
// threads of a warp read consecutive 16-byte packs of shared memory (no bank conflicts), and after
// the last stage the Q states of each column are combined in group order with the reducer's full
// rule (position order for max/min, a fixed order for sums).

template <class R> constexpr size_t strip_combine_bytes() {
    return static_cast<size_t>(kColsConsumers) * (16 / sizeof(typename R::In)) * sizeof(typename R::Local);
}
template <class R> constexpr size_t strip_smem_bytes() {
    return static_cast<size_t>(kStripStages) * kStripStageBytes + 2 * kStripStages * sizeof(uint64_t) +
           strip_combine_bytes<R>();
}

template <class R>
__global__ void __launch_bounds__(kColsThreads, 1) red_cols_strip(const __grid_constant__ CUtensorMap map, RedArgs p) {
    dependent_wait();  // the previous kernel in the stream has completed and its writes are visible
    using T = typename R::In;
    using S = typename R::State;
    using L = typename R::Local;
    constexpr int VE = 16 / static_cast<int>(sizeof(T));  // columns per pack
    constexpr int NS = kStripStages;
    constexpr int M = kStripRows;
    constexpr int kConsumerWarps = kColsConsumers / 32;
    extern __shared__ __align__(128) unsigned char strip_smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(strip_smem + static_cast<size_t>(NS) * kStripStageBytes);
    uint64_t* empty = full + NS;
    L* comb = reinterpret_cast<L*>(empty + NS);
    __shared__ volatile int failed;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < NS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kConsumerWarps);
        }
        mbar_fence_init();
        failed = 0;
    }
    __syncthreads();

    const int PK = p.strip_pk;
    const int Q = kColsConsumers / PK;
    const int RPS = Q * M;
    const int64_t np = p.N / VE;
    const int64_t strips = static_cast<int64_t>(p.aux.d);
    const int K = static_cast<int>(p.K);  // the planner keeps K below 2^31 - 1
    const int64_t c0 = blockIdx.x, cstep = gridDim.x;
    if (warp == kConsumerWarps) {
        // ---- producer
        uint32_t g = 0;
        bool ok = true;
        for (int64_t u = c0; u < p.strip_units && ok; u += cstep) {
            uint64_t b, s;
            p.aux.divmod(static_cast<uint64_t>(u), b, s);
            const int x = static_cast<int>(static_cast<int64_t>(s) * np / strips * VE);
            for (int k = 0; k < K; k += RPS, ++g) {
                const int slot = static_cast<int>(g % NS);
                const bool w = mbar_wait(&empty[slot], ((g / NS) & 1u) ^ 1u);
                if (!__all_sync(0xffffffffu, w)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(RPS * PK * 16));
                    tensor_load_3d(strip_smem + static_cast<size_t>(slot) * kStripStageBytes, &map, x, k,
                                   static_cast<int>(b), &full[slot]);
                }
            }
        }
        if (!ok && lane == 0) {
            note_timeout(p.timeouts);
            failed = 1;
            // let the copies already issued land before the CTA's shared memory goes away
            for (uint32_t i = g > static_cast<uint32_t>(NS) ? g - NS : 0u; i < g; ++i)
                mbar_wait(&full[i % NS], (i / NS) & 1u);
        }
        return;
    }

    // ---- consumers
    const int t = threadIdx.x;
    const int q = t / PK, j = t - q * PK;
    uint32_t g = 0;
    for (int64_t u = c0; u < p.strip_units; u += cstep) {
        uint64_t b, s;
        p.aux.divmod(static_cast<uint64_t>(u), b, s);
        const int64_t p0 = static_cast<int64_t>(s) * np / strips;
        const int64_t p1 = (static_cast<int64_t>(s) + 1) * np / strips;
        const bool active = q < Q && j < p1 - p0;
        L st[VE];
#pragma unroll
        for (int e = 0; e < VE; ++e) st[e] = R::local_init();
        for (int k = 0; k < K; k += RPS, ++g) {
            const int slot = static_cast<int>(g % NS);
            const bool w = !failed && mbar_wait(&full[slot], (g / NS) & 1u);
            if (!__all_sync(0xffffffffu, w)) {
                // give up on the rest: no more waits or folds, but every named barrier below is
                // still met so that the other consumer warps finish too
                if (lane == 0 && !failed) {
                    note_timeout(p.timeouts);
                    failed = 1;
                }
                continue;
            }
            const T* sb = reinterpret_cast<const T*>(strip_smem + static_cast<size_t>(slot) * kStripStageBytes) +
                          static_cast<int64_t>(q * PK + j) * VE;
            const int step = Q * PK * VE;  // elements from one of the thread's rows to its next
            const int r0 = k + q;
            if (active) {
                if (k + RPS <= K) {
                    Pack<T, VE> x[M];
#pragma unroll
                    for (int i = 0; i < M; ++i) x[i] = *reinterpret_cast<const Pack<T, VE>*>(sb + i * step);
#pragma unroll
                    for (int i = 0; i < M; ++i)
#pragma unroll
                        for (int e = 0; e < VE; ++e) R::fold_local(st[e], x[i].v[e], r0 + i * Q);
                } else {
                    for (int i = 0; i < M && r0 + i * Q < K; ++i) {
                        const Pack<T, VE> x = *reinterpret_cast<const Pack<T, VE>*>(sb + i * step);
#pragma unroll
                        for (int e = 0; e < VE; ++e) R::fold_local(st[e], x.v[e], r0 + i * Q);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
        if (u + cstep >= p.strip_units) allow_dependents();  // this CTA's last unit is read
        // combine the row groups' states of each column in group order
        if (active) {
#pragma unroll
            for (int e = 0; e < VE; ++e) comb[(q * PK + j) * VE + e] = st[e];
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kColsConsumers) : "memory");
        const int cols = static_cast<int>(p1 - p0) * VE;
        if (t < cols && !failed) {
            S r = R::widen(comb[t], 0);
            for (int g2 = 1; g2 < Q; ++g2) R::combine(r, R::widen(comb[g2 * PK * VE + t], 0));
            int64_t o1 = 0, o2 = 0;
            if (p.rank_k == 2) {
                o1 = static_cast<int64_t>(b) * p.stride_o[0];
                o2 = static_cast<int64_t>(b) * p.stride_o2[0];
            }
            const int64_t col = p0 * VE + t;
            R::write(p, r, o1 + col, o2 + col);
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kColsConsumers) : "memory");
    }
}

// ------------------------------------------------------------------------------------------------
// Narrow column reductions (4- and 8-byte types): each batch row is a contiguous [K, N] block
// whose rows are at most 1 KiB. A CTA streams whole rows [k0, k1) of one block as
// a flat run of packs: thread t reads pack t, t + M, t + 2M, ... (M = np * lanes, a multiple of
// the np packs of a row), so it always meets column group t % np, in rows t / np, t / np + lanes,
// ... in increasing order, and every warp load is one contiguous 512-byte run. The `lanes`
// threads of a column group are then combined in row order through shared memory; the CTA's
// result is the output, or its split's partial (combined in split order by red_finalize).
template <class R> __global__ void __launch_bounds__(kNarrowBlock) red_cols_narrow(RedArgs p) {
    dependent_wait();  // the previous kernel in the stream has completed and its writes are visible
    allow_dependents();  // one-wave grid: the next kernel (a second pass or the next op) may launch now
    using T = typename R::In;
    using S = typename R::State;
    constexpr int VE = 16 / static_cast<int>(sizeof(T));
    constexpr int U = 4;  // packs in flight per thread
    __shared__ S red[kNarrowBlock * VE];
    const int np = static_cast<int>(p.N / VE);
    const int lanes = kNarrowBlock / np > 0 ? kNarrowBlock / np : 1;
    const int M = np * lanes;  // threads in use
    const int t = threadIdx.x;
    const bool active = t < M;
    const int g = active ? t % np : 0, rl = active ? t / np : 0;
    const int64_t batches = p.kept / p.N;
    const int64_t total = batches * p.split;
    for (int64_t w = blockIdx.x; w < total; w += gridDim.x) {
        uint64_t b, sp;
        p.aux2.divmod(static_cast<uint64_t>(w), b, sp);
        int64_t in_off = 0, o1 = 0, o2 = 0;
        {
            uint64_t bb = b;
            for (int d = p.rank_k - 2; d >= 0; --d) {
                uint64_t q, c;
                p.div_k[d].divmod(bb, q, c);
                in_off += static_cast<int64_t>(c) * p.stride_k[d];
                o1 += static_cast<int64_t>(c) * p.stride_o[d];
                o2 += static_cast<int64_t>(c) * p.stride_o2[d];
                bb = q;
            }
        }
        const int64_t k0 = static_cast<int64_t>(sp) * p.chunk;
        const int64_t k1 = k0 + p.chunk < p.K ? k0 + p.chunk : p.K;
        typename R::Local st[VE];
#pragma unroll
        for (int e = 0; e < VE; ++e) st[e] = R::local_init();
        if (active) {
            const T* base = static_cast<const T*>(p.in) + in_off + g * VE;
            for (int64_t k = k0 + rl; k < k1; k += static_cast<int64_t>(lanes) * U) {
                Pack<T, VE> x[U];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int64_t kk = k + static_cast<int64_t>(u) * lanes;
                    if (kk < k1) x[u] = load_pack<T, VE>(base + kk * p.strideK);
                }
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int64_t kk = k + static_cast<int64_t>(u) * lanes;
                    if (kk < k1) {
                        const int32_t j = static_cast<int32_t>(kk - k0);
#pragma unroll
                        for (int e = 0; e < VE; ++e) R::fold_local(st[e], x[u].v[e], j);
                    }
                }
            }
#pragma unroll
            for (int e = 0; e < VE; ++e) red[t * VE + e] = R::widen(st[e], k0);
        }
        __syncthreads();
        if (active && rl == 0) {
            // thread g combines the lanes of column group g in row-lane order
#pragma unroll
            for (int e = 0; e < VE; ++e) {
                S acc = red[g * VE + e];
                for (int l = 1; l < lanes; ++l) R::combine(acc, red[(l * np + g) * VE + e]);
                const int64_t col = static_cast<int64_t>(g) * VE + e;
                if (p.split == 1) {
                    R::write(p, acc, o1 + col, o2 + col);
                } else {
                    const int64_t kidx = static_cast<int64_t>(b) * p.N + col;
                    static_cast<S*>(p.scratch)[kidx * p.split + static_cast<int64_t>(sp)] = acc;
                }
            }
        }
        __syncthreads();
    }
}

// One thread per output, folding the reduced subspace in row-major order (the CPU's order).
template <class R> __global__ void __launch_bounds__(kRedBlock) red_general_thread(RedArgs p) {
    dependent_wait();  // the previous kernel in the stream has completed and its writes are visible
    allow_dependents();  // one-wave grid: the next kernel (a second pass or the next op) may launch now
    using T = typename R::In;
    using S = typename R::State;
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nthr = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const T* in = static_cast<const T*>(p.in);
    for (int64_t k = tid; k < p.kept; k += nthr) {
        int64_t in_off, o1, o2;
        red_decode_kept(p, static_cast<uint64_t>(k), in_off, o1, o2);
        S st = R::init();
        for (int64_t j = 0; j < p.red; ++j) R::fold(st, in[in_off + red_decode_red(p, j)], j);
        R::write(p, st, o1, o2);
    }
}

// CTAs share one output's reduced range (few outputs, long strided reductions).
template <class R> __global__ void __launch_bounds__(kRedBlock) red_general_cta(RedArgs p) {
    dependent_wait();  // the previous kernel in the stream has completed and its writes are visible
    allow_dependents();  // one-wave grid: the next kernel (a second pass or the next op) may launch now
    using T = typename R::In;
    using S = typename R::State;
    __shared__ S smem[32];
    const T* in = static_cast<const T*>(p.in);
    const int64_t total = p.kept * p.split;
    for (int64_t t = blockIdx.x; t < total; t += gridDim.x) {
        uint64_t k, sp;
        p.aux.divmod(static_cast<uint64_t>(t), k, sp);
        int64_t in_off, o1, o2;
        red_decode_kept(p, k, in_off, o1, o2);
        const int64_t j0 = static_cast<int64_t>(sp) * p.chunk;
        const int64_t j1 = j0 + p.chunk < p.red ? j0 + p.chunk : p.red;
        S st = R::init();
        for (int64_t j = j0 + threadIdx.x; j < j1; j += blockDim.x)
            R::fold(st, in[in_off + red_decode_red(p, static_cast<uint64_t>(j))], j);
        st = block_reduce<R>(st, smem);
        if (threadIdx.x == 0) {
            if (p.split == 1) R::write(p, st, o1, o2);
            else static_cast<S*>(p.scratch)[t] = st;
        }
    }
}

// CTAs share one output's reduced range, whose innermost reduced dim is contiguous (runs of
// shape_r[rank_r - 1] elements, a whole number of 16-byte packs, every run on a 16-byte
// boundary): e.g. a sum over dims 0 and 2 of [64, 1024, 1024]. The output's runs are one sequence
// of packs (aux2 = packs per run); thread t takes packs t, t + 256, ... with 4 in flight,
// decoding each pack's run once, so every load is a 16-byte pack and a warp reads 512 contiguous
// bytes of a run. Each thread folds its elements in increasing position, so the first-index and
// first-NaN rules hold within it and block_reduce combines the threads by position. p.chunk
// counts packs per split.
template <class R> __global__ void __launch_bounds__(kRedBlock) red_runs_cta(RedArgs p) {
    dependent_wait();  // the previous kernel in the stream has completed and its writes are visible
    allow_dependents();  // one-wave grid: the next kernel (a second pass or the next op) may launch now
    using T = typename R::In;
    using S = typename R::State;
    constexpr int V = 16 / static_cast<int>(sizeof(T));
    constexpr int U = 4;
    __shared__ S smem[32];
    const T* in = static_cast<const T*>(p.in);
    const int64_t L = p.shape_r[p.rank_r - 1];
    const int64_t npacks = p.red / V;
    const int64_t total = p.kept * p.split;
    for (int64_t t = blockIdx.x; t < total; t += gridDim.x) {
        uint64_t k, sp;
        p.aux.divmod(static_cast<uint64_t>(t), k, sp);
        int64_t in_off, o1, o2;
        red_decode_kept(p, k, in_off, o1, o2);
        const int64_t q0 = static_cast<int64_t>(sp) * p.chunk;
        const int64_t q1 = q0 + p.chunk < npacks ? q0 + p.chunk : npacks;
        S st = R::init();
        for (int64_t q = q0 + threadIdx.x; q < q1; q += static_cast<int64_t>(blockDim.x) * U) {
            Pack<T, V> x[U];
            int64_t pos[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int64_t qq = q + static_cast<int64_t>(u) * blockDim.x;
                if (qq < q1) {
                    uint64_t r, c;
                    p.aux2.divmod(static_cast<uint64_t>(qq), r, c);
                    const int64_t j = static_cast<int64_t>(r) * L;  // first position of the run
                    pos[u] = j + static_cast<int64_t>(c) * V;
                    x[u] = load_pack<T, V>(in + in_off + red_decode_run(p, r) + static_cast<int64_t>(c) * V);
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int64_t qq = q + static_cast<int64_t>(u) * blockDim.x;
                if (qq < q1) {
#pragma unroll
                    for (int e = 0; e < V; ++e) R::fold(st, x[u].v[e], pos[u] + e);
                }
            }
        }
        st = block_reduce<R>(st, smem);
        if (threadIdx.x == 0) {
            if (p.split == 1) R::write(p, st, o1, o2);
            else static_cast<S*>(p.scratch)[t] = st;
        }
    }
}

// Second pass for few outputs with many partials each (a whole-tensor sum split over every SM):
// one CTA per output; thread t folds partials t, t + 256, ... in order, then a fixed-shape tree
// (warp shuffles, then the warps' results) combines the threads. The shape depends only on the
// split count, so results are run-to-run identical; the partial loads overlap instead of forming
// one thread's chain of dependent loads.
template <class R> __global__ void __launch_bounds__(kRedBlock) red_finalize_cta(RedArgs p) {
    dependent_wait();  // the first pass has completed and its partials are visible
    allow_dependents();  // small kernel: the next one in the stream may launch during it
    using S = typename R::State;
    __shared__ S smem[kRedBlock / 32];
    const S* part = static_cast<const S*>(p.scratch);
    for (int64_t k = blockIdx.x; k < p.kept; k += gridDim.x) {
        S st = R::init();
        for (int s = threadIdx.x; s < p.split; s += blockDim.x) R::combine(st, part[k * p.split + s]);
        st = block_reduce<R>(st, smem);
        if (threadIdx.x == 0) {
            int64_t in_off, o1, o2;
            red_decode_kept(p, static_cast<uint64_t>(k), in_off, o1, o2);
            R::write(p, st, o1, o2);
        }
    }
}

// Second pass: combine the `split` partials of each output in split order.
template <class R> __global__ void __launch_bounds__(kRedBlock) red_finalize(RedArgs p) {
    dependent_wait();  // the first pass has completed and its partials are visible
    allow_dependents();  // small kernel: the next one in the stream may launch during it
    using S = typename R::State;
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nthr = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const S* part = static_cast<const S*>(p.scratch);
    for (int64_t k = tid; k < p.kept; k += nthr) {
        S st = part[k * p.split];
        for (int s = 1; s < p.split; ++s) R::combine(st, part[k * p.split + s]);
        int64_t in_off, o1, o2;
        red_decode_kept(p, static_cast<uint64_t>(k), in_off, o1, o2);
        R::write(p, st, o1, o2);
    }
}

// ------------------------------------------------------------------------------------------------
// launcher

// Outer-path vector width for element type T.
template <class T> constexpr int outer_vec() { return sizeof(T) >= 8 ? 2 : 4; }

template <class R>
int launch_reduction(RedPlan& plan, void* scratch, size_t scratch_bytes, size_t need,
                     cudaStream_t st) {
    RedArgs& a = plan.args;
    if (plan.path == RedPath::Empty) return CTB_OK;
    if (need > 0) {
        if (scratch == nullptr || scratch_bytes < need)
            return fail(CTB_ERR_SCRATCH, "scratch buffer too small: need " + std::to_string(need) +
                                             " bytes, got " + std::to_string(scratch_bytes));
        a.scratch = scratch;
    }
    int launches = 1;
    switch (plan.path) {
    case RedPath::Inner:
        if (plan.warp_rows) {
            note_reduction_kernel(plan.row_group > 1 ? "red_inner_group" : "red_inner_warp");
            if (plan.row_group == 4) launch_dependent(red_inner_group<R, 4>, plan.grid, kRedBlock, 0, st, a);
            else if (plan.row_group == 2) launch_dependent(red_inner_group<R, 2>, plan.grid, kRedBlock, 0, st, a);
            else launch_dependent(red_inner_warp<R>, plan.grid, kRedBlock, 0, st, a);
        } else {
            note_reduction_kernel("red_inner_cta");
            launch_dependent(red_inner_cta<R>, plan.grid, kRedBlock, 0, st, a);
        }
        break;
    case RedPath::Outer: {
        using T = typename R::In;
        if constexpr (sizeof(T) >= 4) {
            if (plan.narrow) {
                note_reduction_kernel("red_cols_narrow");
                launch_dependent(red_cols_narrow<R>, plan.grid, kNarrowBlock, 0, st, a);
                break;
            }
        }
        if constexpr (sizeof(T) >= 4) {
            if (plan.strip) {
                note_reduction_kernel("red_cols_strip");
                launch_dependent(red_cols_strip<R>, plan.grid, kColsThreads, strip_smem_bytes<R>(), st,
                                 plan.strip_map, a);
                break;
            }
        }
        if (plan.bulk) {
            note_reduction_kernel("red_cols_bulk");
            launch_dependent(red_cols_bulk<R>, plan.grid, kColsThreads, cols_smem_bytes(), st, a);
            if (int rc = check_launch("reduction")) return rc;
            if (plan.bulk_fixup) {
                const cudaError_t e = launch_dependent(red_cols_finalize<R>, grid_for((a.kept + 31) / 32, 8),
                                                       32 * kColsFixGroups, 0, st, a);
                if (e != cudaSuccess) return fail(CTB_ERR_CUDA, std::string("reduction: ") + cudaGetErrorString(e));
                ++launches;
            }
            break;
        }
        constexpr int VMAX = outer_vec<T>();
        note_reduction_kernel("red_outer");
        if (plan.col_tile == 32 * VMAX) launch_dependent(red_outer<R, VMAX>, plan.grid, kOuterBlock, 0, st, a);
        else launch_dependent(red_outer<R, 1>, plan.grid, kOuterBlock, 0, st, a);
        break;
    }
    case RedPath::General:
        note_reduction_kernel(plan.warp_rows ? "red_general_thread" : plan.runs ? "red_runs_cta" : "red_general_cta");
        if (plan.warp_rows) launch_dependent(red_general_thread<R>, plan.grid, kRedBlock, 0, st, a);
        else if (plan.runs) launch_dependent(red_runs_cta<R>, plan.grid, kRedBlock, 0, st, a);
        else launch_dependent(red_general_cta<R>, plan.grid, kRedBlock, 0, st, a);
        break;
    default:
        break;
    }
    if (a.split > 1) {
        if (int rc = check_launch("reduction")) return rc;
        const cudaError_t e =
            a.split >= 64 && a.kept <= static_cast<int64_t>(sm_count()) * 8
                ? launch_dependent(red_finalize_cta<R>, grid_for(a.kept, 8), kRedBlock, 0, st, a)
                : launch_dependent(red_finalize<R>, grid_for((a.kept + kRedBlock - 1) / kRedBlock, 8), kRedBlock,
                                   0, st, a);
        if (e != cudaSuccess) return fail(CTB_ERR_CUDA, std::string("reduction: ") + cudaGetErrorString(e));
        ++launches;
    }
    count_launch(launches);
    return check_launch("reduction");
}

// Whether the Outer strip kernel may use V-wide loads for this plan.
inline bool outer_vec_ok(const RedPlan& plan, int elem_bytes, int V) {
    const RedArgs& a = plan.args;
    if (plan.path != RedPath::Outer) return false;
    const int bytes = elem_bytes * V;
    if (reinterpret_cast<uintptr_t>(a.in) % bytes) return false;
    if (a.N % V || a.strideK % V) return false;
    for (int d = 0; d < a.rank_k - 1; ++d)
        if (a.stride_k[d] % V) return false;
    return true;
}

// Whether the bulk column kernel can take this Outer plan: every row of every tile starts on a
// 16-byte boundary and every row copy is a whole number of 16-byte chunks; positions within the
// reduced dim fit the kernel's 32-bit offsets.
inline bool cols_bulk_ok(const RedPlan& plan, int elem_bytes) {
    const RedArgs& a = plan.args;
    if (plan.path != RedPath::Outer) return false;
    if (reinterpret_cast<uintptr_t>(a.in) % 16) return false;
    if ((a.N * elem_bytes) % 16 || (a.strideK * elem_bytes) % 16) return false;
    for (int d = 0; d < a.rank_k - 1; ++d)
        if ((a.stride_k[d] * elem_bytes) % 16) return false;
    // at least an eighth of the consumer threads busy (rows of 512 B or more); narrower strips
    // go to red_outer
    if (a.N * elem_bytes < kColsRowBytes / 8) return false;
    return a.K < (int64_t(1) << 31) - 1;
}

// Whether the narrow column kernel can take this Outer plan: each batch row is one contiguous
// [K, N] block (rows back to back) of rows of at most 1 KiB, 16-byte aligned.
inline bool cols_narrow_ok(const RedPlan& plan, int elem_bytes) {
    const RedArgs& a = plan.args;
    if (plan.path != RedPath::Outer) return false;
    if (reinterpret_cast<uintptr_t>(a.in) % 16) return false;
    if ((a.N * elem_bytes) % 16 || a.strideK != a.N) return false;
    // rows up to 1 KiB (four or more threads a column group); wider rows stream better through
    // the bulk kernel (argmax over 65536 x 1024 floats: 53 us bulk against 74 us here)
    if (a.N * elem_bytes > 1024) return false;
    for (int d = 0; d < a.rank_k - 1; ++d)
        if ((a.stride_k[d] * elem_bytes) % 16) return false;
    return a.K < (int64_t(1) << 31) - 1;
}

// Whether the strip column kernel can take this Outer plan: at most one batch dim, the input a
// [batch, K, N] tensor a tensor map can describe (16-byte aligned base, row and batch strides
// whole 16-byte multiples, batches after one another), rows of at least kStripMinK and positions
// that fit the kernel's 32-bit row offsets. Whether the strips come out wide enough is the
// planner's call (strip_geometry).
inline bool cols_strip_ok(const RedPlan& plan, int elem_bytes) {
    const RedArgs& a = plan.args;
    if (plan.path != RedPath::Outer || a.rank_k > 2) return false;
    if (reinterpret_cast<uintptr_t>(a.in) % 16) return false;
    if ((a.N * elem_bytes) % 16 || (a.strideK * elem_bytes) % 16 || a.strideK < a.N) return false;
    if (a.rank_k == 2 && ((a.stride_k[0] * elem_bytes) % 16 || a.stride_k[0] < a.K * a.strideK)) return false;
    return a.K >= kStripMinK && a.K < (int64_t(1) << 31) - 1 && a.N < (int64_t(1) << 31) &&
           a.kept / a.N < (int64_t(1) << 31);
}

// Encodes plan.strip_map for a planned strip reduction: the input as a [batch, K, N] tensor of
// elem_bytes-sized elements, a box of one strip (strip_pk packs) by one stage of rows. False if the
// driver's encoder is missing or refuses the tensor.
bool encode_strip_map(RedPlan& plan, int elem_bytes);

// Address of this device's timed-out-wait counter (async.cu); null if it cannot be had.
unsigned long long* wait_timeout_counter();

// Lets red_cols_bulk<R> use its dynamic shared memory on the current device (once per device).
template <class R> bool cols_bulk_ready() {
    static std::mutex mu;
    static signed char state[64] = {};  // 0 unknown, 1 ready, -1 unavailable
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return false;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (state[dev] == 0) {
        const cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(&red_cols_bulk<R>),
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(cols_smem_bytes()));
        if (e != cudaSuccess) cudaGetLastError();
        state[dev] = e == cudaSuccess ? 1 : -1;
    }
    return state[dev] == 1;
}

// Lets red_cols_strip<R> use its dynamic shared memory on the current device (once per device).
template <class R> bool cols_strip_ready() {
    static std::mutex mu;
    static signed char state[64] = {};  // 0 unknown, 1 ready, -1 unavailable
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return false;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (state[dev] == 0) {
        const cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(&red_cols_strip<R>),
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(strip_smem_bytes<R>()));
        if (e != cudaSuccess) cudaGetLastError();
        state[dev] = e == cudaSuccess ? 1 : -1;
    }
    return state[dev] == 1;
}

// Plans + sizes a reduction for reducer R; returns scratch bytes via `need`.
template <class R>
int plan_for(const ctb_view* in, const ctb_view* out, const ctb_view* out2, uint32_t mask,
             RedPlan& plan, size_t& need) {
    using T = typename R::In;
    int rc = plan_reduction(in, out, out2, mask, plan);
    if (rc) return rc;
    constexpr int V = outer_vec<T>();
    const bool vec_ok = outer_vec_ok(plan, sizeof(T), V);
    RedOcc occ;
    if constexpr (sizeof(T) >= 4) {  // 1-byte columns: 16 chains a thread would not fit
        if (cols_narrow_ok(plan, sizeof(T)))
            occ.cols_narrow = resident_ctas(reinterpret_cast<const void*>(&red_cols_narrow<R>), kNarrowBlock);
    }
    if constexpr (sizeof(T) >= 4) {  // narrower types: 8 or 16 chains a thread, compute-bound
        if (occ.cols_narrow == 0 && cols_strip_ok(plan, sizeof(T)) && cols_strip_ready<R>()) {
            plan.args.timeouts = wait_timeout_counter();
            if (plan.args.timeouts) {
                occ.cols_strip = resident_ctas(reinterpret_cast<const void*>(&red_cols_strip<R>), kColsThreads,
                                               strip_smem_bytes<R>());
                occ.strip_pk_max = 256 / (16 / static_cast<int>(sizeof(T)));
            }
        }
    }
    if (occ.cols_narrow == 0 && cols_bulk_ok(plan, sizeof(T)) && cols_bulk_ready<R>()) {
        plan.args.timeouts = wait_timeout_counter();
        if (plan.args.timeouts)
            occ.cols_bulk = resident_ctas(reinterpret_cast<const void*>(&red_cols_bulk<R>), kColsThreads,
                                          cols_smem_bytes());
    }
    occ.inner_cta = resident_ctas(reinterpret_cast<const void*>(&red_inner_cta<R>), kRedBlock);
    occ.inner_warp = resident_ctas(reinterpret_cast<const void*>(&red_inner_warp<R>), kRedBlock);
    occ.outer = vec_ok ? resident_ctas(reinterpret_cast<const void*>(&red_outer<R, V>), kOuterBlock)
                       : resident_ctas(reinterpret_cast<const void*>(&red_outer<R, 1>), kOuterBlock);
    occ.general_cta = resident_ctas(reinterpret_cast<const void*>(&red_general_cta<R>), kRedBlock);
    occ.runs = resident_ctas(reinterpret_cast<const void*>(&red_runs_cta<R>), kRedBlock);
    need = finish_reduction_plan(plan, sizeof(T), sizeof(typename R::State), vec_ok ? V : 1, occ);
    if (plan.strip && !encode_strip_map(plan, sizeof(T))) {
        occ.cols_strip = 0;  // the bulk kernel (or the register kernel) takes it instead
        need = finish_reduction_plan(plan, sizeof(T), sizeof(typename R::State), vec_ok ? V : 1, occ);
    }
    return CTB_OK;
}

}  // namespace ctb
