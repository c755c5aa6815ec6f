// fused_rows.cu — one pass over a row-major matrix that computes an elementwise chain and reduces
// its result two ways in the epilogue:
//     y = op2(op1(a, b), c)              (written, bit-identical to the two eager ops)
//     idx[row] = arg{min,max}(y[row, :]) (first index on ties, first NaN wins)
//     partial  = sum(y) in float64       (deterministic: fixed per-CTA order, then CTA order)
// a is [R, C] with unit inner stride; b and c are [C] rows broadcast over R (or 0-d scalars).
// One warp per row, persistent grid of one wave; each lane keeps its running extreme with a strict
// compare (so its first occurrence wins without carrying the index through every compare), and the
// lanes' (value, index) states are combined by warp shuffles with the full tie/NaN rule of
// src/ops/reduction_functors.h:55-110. Reads a once and writes y once: the eager sequence
// (chain, then sum, then argmin) reads y twice more.
//
// Across GPUs (ctb_chain_rows_allsum): the last CTA to finish (a ticket in this rank's peer
// workspace, reset by that CTA) also sums the per-CTA partials into the rank's partial, stores it
// over NVLink into slot `rank` of every rank's workspace (an IPC mapping of each peer's memory)
// with the call's epoch, waits until every rank's slot in its own workspace carries that epoch,
// and adds the slots in rank order: the whole-job sum, on every rank, from the one launch. The
// waits are bounded in time; a wait that runs out is counted (ctb_wait_timeouts), recorded in the
// workspace (ctb_peer_status) and leaves NaN as the sum.
#include <limits>

#include "async_copy.cuh"
#include "common.cuh"
#include "peer.cuh"
#include "plan.cuh"

namespace ctb {

struct FusedRowsArgs {
    const void* a;
    const void* b;
    const void* c;
    void* y;          // may be null
    int64_t* idx;     // may be null
    double* partials; // per-CTA sums (scratch), may be null
    int64_t rows, cols;
    int64_t a_row_stride, y_row_stride, idx_stride;
    int b_bcast, c_bcast;  // 1: b/c is a 0-d scalar (stride 0 along the row)
    int c_is_b;
    int is_max;
    // cross-GPU sum (ctb_chain_rows_allsum); peers == nullptr otherwise
    PeerWorkspace* const* peers;  // device array of every rank's workspace (this rank's own at [rank])
    int rank, world;
    uint64_t epoch;
    uint64_t timeout_ns;
    void* out_sum;         // 0-d float32/float64
    int out_sum_dtype;
    double* out_parts;     // [world] rank partials, may be null
    unsigned long long* timeouts;
};

// Sum of n per-CTA partials by one 256-thread block: thread t adds partials t, t + 256, ... in
// order, then a fixed tree (warp shuffles, then the 8 warps' sums in order). Result in thread 0.
// The shape depends only on n, so the sum is run-to-run identical, and the same on the one-GPU
// (fused_rows_combine) and cross-GPU (last CTA) paths.
__device__ __forceinline__ double tree_sum_256(const double* partials, int n, double* sm8) {
    double s = 0.0;
    for (int i = threadIdx.x; i < n; i += 256) s = __dadd_rn(s, __ldcg(partials + i));
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) s = __dadd_rn(s, __shfl_xor_sync(0xffffffffu, s, m));
    if ((threadIdx.x & 31) == 0) sm8[threadIdx.x >> 5] = s;
    __syncthreads();
    double t = 0.0;
    if (threadIdx.x == 0)
        for (int w = 0; w < 8; ++w) t = __dadd_rn(t, sm8[w]);
    return t;
}

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Cross-GPU epilogue, run by every thread of the last CTA of this rank's launch (256 threads).
// Slots are double-buffered by epoch parity and a slot is accepted only when it carries exactly
// this call's epoch (peer.cuh). A wait that runs out leaves NaN in out_sum (and in the missing
// ranks' entries of out_parts), records the epoch in the workspace's failed_epoch and is counted.
__device__ void allsum_epilogue(const FusedRowsArgs& p) {
    __shared__ double sm8[8];
    __shared__ double rank_sum[kPeerMaxRanks];
    __shared__ int ok_all;
    const double mine = tree_sum_256(p.partials, static_cast<int>(gridDim.x), sm8);
    __shared__ double mine_sh;
    if (threadIdx.x == 0) {
        mine_sh = mine;
        ok_all = 1;
    }
    __syncthreads();
    const int g = threadIdx.x;
    const int par = static_cast<int>(p.epoch & 1u);
    if (g < p.world) {
        // publish: value, then the epoch that marks it valid, as a system-scope release store (it
        // orders this thread's value store before it for every observer, the peers included)
        PeerSlot* dst = &p.peers[g]->slots[par][p.rank];
        *reinterpret_cast<volatile double*>(&dst->value) = mine_sh;
        st_release_sys(&dst->epoch, p.epoch);
    }
    if (g < p.world) {
        // wait for rank g's value of this epoch in this rank's own workspace
        PeerSlot* src = &p.peers[p.rank]->slots[par][g];
        bool ok = ld_acquire_sys(&src->epoch) == p.epoch;
        if (!ok) {
            const uint64_t t0 = global_ns();
            while (!(ok = ld_acquire_sys(&src->epoch) == p.epoch))
                if (global_ns() - t0 > p.timeout_ns) break;
        }
        if (ok) rank_sum[g] = *reinterpret_cast<volatile const double*>(&src->value);
        else {
            rank_sum[g] = __longlong_as_double(0x7ff8000000000000ll);
            atomicExch(&ok_all, 0);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        PeerWorkspace* me = p.peers[p.rank];
        double s = 0.0;
        for (int r = 0; r < p.world; ++r) {  // rank order
            s = __dadd_rn(s, rank_sum[r]);
            if (p.out_parts) p.out_parts[r] = rank_sum[r];
        }
        if (!ok_all) {
            s = __longlong_as_double(0x7ff8000000000000ll);
            me->failed_epoch = p.epoch;
            note_timeout(p.timeouts);
        } else {
            me->done_epoch = p.epoch;
        }
        if (p.out_sum_dtype == CTB_FLOAT32) *static_cast<float*>(p.out_sum) = static_cast<float>(s);
        else *static_cast<double*>(p.out_sum) = s;
        me->trace[p.epoch % kPeerTraceSlots][kTraceExchanged] = global_ns();
    }
}

template <class T> __device__ __forceinline__ T extreme_ident(bool is_max) {
    return is_max ? -std::numeric_limits<T>::infinity() : std::numeric_limits<T>::infinity();
}

// op2(op1(x, b), c), or op1(x, b) alone when OP2 is kOpNone (ctb_binary on row-broadcast rows).
template <int OP1, int OP2, class T> __device__ __forceinline__ T chain_apply(T x, T b, T c) {
    if constexpr (OP2 == kOpNone) return BinOp<OP1>::template apply<T>(x, b);
    else return BinOp<OP2>::template apply<T>(BinOp<OP1>::template apply<T>(x, b), c);
}

// STAGE: b and c are copied once per CTA into shared memory (a 0-d scalar is expanded to a row),
// so the per-element reads of the broadcast row never hold registers across the latency of the
// loads of a; without STAGE (rows too long for shared memory) they are read through L1.
// RED = false: the chain alone (y only; no row extreme, no sum), for ctb_binary_chain on
// row-broadcast operands.
template <int OP1, int OP2, class T, int V, bool STAGE, bool RED = true>
__global__ void __launch_bounds__(256) fused_rows_kernel(FusedRowsArgs p) {
    dependent_wait();  // the previous kernel in the stream has completed and its writes are visible
    constexpr int U = 4;
    extern __shared__ __align__(16) unsigned char fr_smem[];
    const int lane = threadIdx.x & 31;
    const int C = static_cast<int>(p.cols);
    const T* __restrict__ B = static_cast<const T*>(p.b);
    const T* __restrict__ Cc = static_cast<const T*>(p.c);
    if constexpr (STAGE) {
        T* sb = reinterpret_cast<T*>(fr_smem);
        constexpr int kPad = 16 / sizeof(T);  // keep the second row 16-byte aligned
        T* sc = sb + (p.c_is_b ? 0 : (C + kPad - 1) / kPad * kPad);
        const T b0 = p.b_bcast ? B[0] : T(0);
        const T c0 = p.c_bcast ? Cc[0] : T(0);
        // A row read as 16-byte packs, eight per thread in flight before any is stored, so the
        // staging costs one round trip to L2 instead of one per element.
        auto stage_row = [&](T* dst, const T* src, bool bcast, T v0) {
            constexpr int PV = 16 / static_cast<int>(sizeof(T));
            if (!bcast && V > 1) {  // V > 1: the rows are 16-byte aligned (pack path)
                const int np = C / PV;
                for (int j0 = threadIdx.x; j0 < np; j0 += 8 * blockDim.x) {
                    Pack<T, PV> x[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u)
                        if (j0 + u * static_cast<int>(blockDim.x) < np)
                            x[u] = load_pack<T, PV>(src + (j0 + u * static_cast<int>(blockDim.x)) * PV);
#pragma unroll
                    for (int u = 0; u < 8; ++u)
                        if (j0 + u * static_cast<int>(blockDim.x) < np)
                            *reinterpret_cast<Pack<T, PV>*>(dst + (j0 + u * static_cast<int>(blockDim.x)) * PV) = x[u];
                }
                for (int j = np * PV + threadIdx.x; j < C; j += blockDim.x) dst[j] = src[j];
            } else {
                for (int j = threadIdx.x; j < C; j += blockDim.x) dst[j] = bcast ? v0 : src[j];
            }
        };
        stage_row(sb, B, p.b_bcast != 0, b0);
        if (!p.c_is_b) stage_row(sc, Cc, p.c_bcast != 0, c0);
        __syncthreads();
        B = sb;
        Cc = sc;
    }
    if (RED && p.peers && blockIdx.x == 0 && threadIdx.x == 0)
        p.peers[p.rank]->trace[p.epoch % kPeerTraceSlots][kTraceStart] = global_ns();
    const bool b_row = STAGE || !p.b_bcast;
    const bool c_row = STAGE || !p.c_bcast;
    const T* __restrict__ A = static_cast<const T*>(p.a);
    T* __restrict__ Y = static_cast<T*>(p.y);
    const bool is_max = p.is_max != 0;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    const int nv = C / V;  // whole packs per row (V == 1 when rows are not pack-aligned)
    double sum = 0.0;

    // One element of the chain, folded into the row's extreme and the thread's sum.
    auto element = [&](T xv, T bb, T cc, int j, T& best, int& bidx) -> T {
        const T yv = chain_apply<OP1, OP2, T>(xv, bb, cc);
        if constexpr (RED) {
            sum = __dadd_rn(sum, static_cast<double>(yv));
            const bool repl = (best == best) && ((yv != yv) || (is_max ? yv > best : yv < best));
            if (repl) {
                best = yv;
                bidx = j;
            }
        }
        return yv;
    };
    // Packs [v0 + 32u] of one row: compute, fold, store. The lean form (tag true) is the common
    // case with every check hoisted out: b a staged row, c the same row, y written, and the row a
    // whole number of batches; at 16 warps per SM the instructions per element set the pace.
    auto do_packs = [&](auto lean_tag, const Pack<T, V>* xa, int v0, T* yr, T& best, int& bidx) {
        constexpr bool L = decltype(lean_tag)::value;
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int v = v0 + u * 32;
            if (L || v < nv) {
                Pack<T, V> xb, xc, o;
                if (L || b_row) xb = *reinterpret_cast<const Pack<T, V>*>(B + v * V);
                if (!L && !p.c_is_b && c_row) xc = *reinterpret_cast<const Pack<T, V>*>(Cc + v * V);
#pragma unroll
                for (int e = 0; e < V; ++e) {
                    const T bb = (L || b_row) ? xb.v[e] : B[0];
                    const T cc = (L || p.c_is_b) ? bb : (c_row ? xc.v[e] : Cc[0]);
                    o.v[e] = element(xa[u].v[e], bb, cc, v * V + e, best, bidx);
                }
                if (L || yr) store_pack<T, V>(yr + static_cast<int64_t>(v) * V, o);
            }
        }
    };
    // The row's columns past its last whole pack, then its extreme: lanes combined with NaN first
    // (lowest index), then the extreme value, then the lower index. A lane that saw only +-inf
    // (the min/max identity) keeps index -1 = "empty"; a row of nothing else gives index 0.
    auto finish_row = [&](int64_t row, const T* ar, T* yr, T& best, int& bidx) {
        for (int j = nv * V + lane; j < C; j += 32) {
            const T bb = b_row ? B[j] : B[0];
            const T cc = p.c_is_b ? bb : (c_row ? Cc[j] : Cc[0]);
            const T yv = element(ar[j], bb, cc, j, best, bidx);
            if (yr) yr[j] = yv;
        }
        if (RED && p.idx) {
#pragma unroll
            for (int m = 16; m >= 1; m >>= 1) {
                const T ov = __shfl_xor_sync(0xffffffffu, best, m);
                const int oi = __shfl_xor_sync(0xffffffffu, bidx, m);
                bool take;
                if (oi < 0) take = false;
                else if (bidx < 0) take = true;
                else {
                    const bool an = best != best, bn = ov != ov;
                    if (an || bn) take = an ? (bn && oi < bidx) : true;
                    else if (is_max ? ov > best : ov < best) take = true;
                    else take = (ov == best) && oi < bidx;
                }
                if (take) {
                    best = ov;
                    bidx = oi;
                }
            }
            if (lane == 0) p.idx[row * p.idx_stride] = bidx < 0 ? 0 : bidx;
        }
    };

    if constexpr (V > 1 && !RED) {
        // The chain alone (no reductions), software-pipelined over the warp's batches (U packs a
        // lane of one row), row after row: the loads of the next batch, in this row or the next,
        // are issued before the stores of this one, so every warp keeps reads in flight while it
        // writes. With 16 warps per SM (the grid plan_fused picks for rows of a whole batch or
        // more) it streams at the copy rate: y = (x - r) * r over [262144, 8192] float32 on B200,
        // 2585 us against 2788-2802 us for the row loop below at 32 warps per SM, and a device
        // copy of the same bytes 2578 us. The kernel with its reductions keeps the row loop:
        // pipelined at 16 warps per SM its extra instructions (the float64 sum and the row
        // extreme) left it issue-bound at 3.1-3.2 ms, against 2.7 ms for the row loop at 32.
        const int per_row = nv > 32 * U ? (nv + 32 * U - 1) / (32 * U) : 1;  // batches per row
        // the lean batch body: b a staged row, c the same row, y written, whole batches
        const bool lean = STAGE && p.c_is_b && !p.b_bcast && Y != nullptr && nv % (32 * U) == 0;
        const int64_t my_rows = warp < p.rows ? (p.rows - warp + nwarps - 1) / nwarps : 0;
        const int64_t nb = my_rows * per_row;
        int64_t row = warp, nrow = warp;
        int k = 0, nk = 0;
        auto advance = [&](int64_t& r, int& b) {
            if (++b == per_row) {
                b = 0;
                r += nwarps;
            }
        };
        auto load_batch = [&](Pack<T, V>* xa, int64_t r, int b) {
            const T* ar = A + r * p.a_row_stride;
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int v = b * 32 * U + u * 32 + lane;
                if (lean || v < nv) xa[u] = load_pack<T, V>(ar + static_cast<int64_t>(v) * V);
            }
        };
        Pack<T, V> xa[U];
        if (nb > 0) load_batch(xa, row, 0);
        advance(nrow, nk);
        T best = extreme_ident<T>(is_max);
        int bidx = -1;
        for (int64_t t = 0; t < nb; ++t) {
            const bool more = t + 1 < nb;
            Pack<T, V> nx[U];
            if (more) load_batch(nx, nrow, nk);
            T* yr = Y ? Y + row * p.y_row_stride : nullptr;
            const int v0 = k * 32 * U + lane;
            if (lean) do_packs(std::true_type{}, xa, v0, yr, best, bidx);
            else do_packs(std::false_type{}, xa, v0, yr, best, bidx);
            if (k == per_row - 1) {
                finish_row(row, A + row * p.a_row_stride, yr, best, bidx);
                best = extreme_ident<T>(is_max);
                bidx = -1;
            }
            if (more) {
#pragma unroll
                for (int u = 0; u < U; ++u) xa[u] = nx[u];
            }
            row = nrow;
            k = nk;
            advance(nrow, nk);
        }
    } else {
        for (int64_t row = warp; row < p.rows; row += nwarps) {
            const T* ar = A + row * p.a_row_stride;
            T* yr = Y ? Y + row * p.y_row_stride : nullptr;
            T best = extreme_ident<T>(is_max);
            int bidx = -1;
            for (int v0 = lane; v0 < nv; v0 += 32 * U) {
                Pack<T, V> xa[U];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int v = v0 + u * 32;
                    if (v < nv) xa[u] = load_pack<T, V>(ar + static_cast<int64_t>(v) * V);
                }
                do_packs(std::false_type{}, xa, v0, yr, best, bidx);
            }
            finish_row(row, ar, yr, best, bidx);
        }
    }
    // the next kernel in the stream may launch now (it waits for this one to complete before it
    // touches memory): its launch overlaps this kernel's partial sums and cross-GPU exchange
    allow_dependents();
    if (RED && p.partials) {
        __shared__ double sm[8];
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) sum = __dadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, m));
        if (lane == 0) sm[threadIdx.x >> 5] = sum;
        __syncthreads();
        if (threadIdx.x == 0) {
            double s = 0.0;
            for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) s = __dadd_rn(s, sm[w]);
            p.partials[blockIdx.x] = s;
        }
        if (p.peers) {
            // the last CTA to finish takes the cross-GPU epilogue
            __shared__ int last;
            if (threadIdx.x == 0) {
                __threadfence();
                PeerWorkspace* me = p.peers[p.rank];
                const unsigned tk = atomicAdd(&me->ticket, 1u);
                last = tk == gridDim.x - 1;
                uint64_t* tr = me->trace[p.epoch % kPeerTraceSlots];
                if (tk == 0) tr[kTraceFirstDone] = global_ns();
                if (last) {
                    me->ticket = 0u;  // every CTA has taken its ticket: ready for the next call
                    tr[kTraceLastDone] = global_ns();
                }
            }
            __syncthreads();
            if (last) {
                __threadfence();
                allsum_epilogue(p);
            }
        }
    }
}

// Sum of the per-CTA partials (tree_sum_256: the loads overlap, the order is fixed).
__global__ void __launch_bounds__(256) fused_rows_combine(const double* partials, int n, double* out) {
    dependent_wait();  // the previous kernel in the stream has completed and its writes are visible
    allow_dependents();  // small kernel: the next one in the stream may launch during it
    __shared__ double sm[8];
    const double t = tree_sum_256(partials, n, sm);
    if (threadIdx.x == 0) *out = t;
}

template <int OP1, int OP2, class T>
static const void* pick_kernel(bool vec, bool stage, bool red) {
    constexpr int V = 16 / sizeof(T);
    if (!red) return reinterpret_cast<const void*>(&fused_rows_kernel<OP1, OP2, T, V, true, false>);
    if (stage)
        return vec ? reinterpret_cast<const void*>(&fused_rows_kernel<OP1, OP2, T, V, true>)
                   : reinterpret_cast<const void*>(&fused_rows_kernel<OP1, OP2, T, 1, true>);
    return vec ? reinterpret_cast<const void*>(&fused_rows_kernel<OP1, OP2, T, V, false>)
               : reinterpret_cast<const void*>(&fused_rows_kernel<OP1, OP2, T, 1, false>);
}

// red = false only with vec && stage (fused_chain_rows checks both before it launches).
template <int OP1, int OP2, class T>
static void launch_typed(bool vec, bool stage, bool red, unsigned grid, size_t smem, const FusedRowsArgs& p,
                         cudaStream_t st) {
    constexpr int V = 16 / sizeof(T);
    if (!red) {
        launch_dependent(fused_rows_kernel<OP1, OP2, T, V, true, false>, grid, 256, smem, st, p);
        return;
    }
    if (stage) {
        if (vec) launch_dependent(fused_rows_kernel<OP1, OP2, T, V, true>, grid, 256, smem, st, p);
        else launch_dependent(fused_rows_kernel<OP1, OP2, T, 1, true>, grid, 256, smem, st, p);
    } else {
        if (vec) launch_dependent(fused_rows_kernel<OP1, OP2, T, V, false>, grid, 256, 0, st, p);
        else launch_dependent(fused_rows_kernel<OP1, OP2, T, 1, false>, grid, 256, 0, st, p);
    }
}

template <class T>
static void launch_ops(int op1, int op2, bool vec, bool stage, bool red, unsigned grid, size_t smem,
                       const FusedRowsArgs& p, cudaStream_t st, const void** fn_out) {
#define CTB_FR(O1, O2)                                                            \
    if (op1 == O1 && op2 == O2) {                                                 \
        if (fn_out) *fn_out = pick_kernel<O1, O2, T>(vec, stage, red);            \
        else launch_typed<O1, O2, T>(vec, stage, red, grid, smem, p, st);         \
        return;                                                                   \
    }
    CTB_FR(CTB_SUB, CTB_MUL) CTB_FR(CTB_ADD, CTB_MUL) CTB_FR(CTB_MUL, CTB_ADD) CTB_FR(CTB_SUB, CTB_DIV)
    CTB_FR(CTB_ADD, CTB_ADD) CTB_FR(CTB_SUB, CTB_SUB) CTB_FR(CTB_MUL, CTB_MUL) CTB_FR(CTB_DIV, CTB_DIV)
    CTB_FR(CTB_ADD, CTB_SUB) CTB_FR(CTB_ADD, CTB_DIV) CTB_FR(CTB_SUB, CTB_ADD) CTB_FR(CTB_MUL, CTB_SUB)
    CTB_FR(CTB_MUL, CTB_DIV) CTB_FR(CTB_DIV, CTB_ADD) CTB_FR(CTB_DIV, CTB_SUB) CTB_FR(CTB_DIV, CTB_MUL)
    CTB_FR(CTB_ADD, kOpNone) CTB_FR(CTB_SUB, kOpNone) CTB_FR(CTB_MUL, kOpNone) CTB_FR(CTB_DIV, kOpNone)
#undef CTB_FR
}

// Largest staged footprint (b and c rows) that still leaves room for two CTAs per SM.
constexpr size_t kMaxStageBytes = 96 * 1024;
// Shared memory a CTA of the pipelined loop asks for at least: two fit in an SM's 228 KiB, three
// do not.
constexpr size_t kPipeSmemBytes = 80 * 1024;

// Validation + planning shared by the scratch query and the launch. Returns the grid.
static int plan_fused(int op1, int op2, const ctb_view* a, const ctb_view* b, const ctb_view* c,
                      const ctb_view* y, int row_op, const ctb_view* idx, FusedRowsArgs& p,
                      bool& vec, bool& stage, size_t& smem, unsigned& grid, bool red = true) {
    if (op1 < CTB_ADD || op1 > CTB_DIV || ((op2 < CTB_ADD || op2 > CTB_DIV) && !(op2 == kOpNone && !red)))
        return fail(CTB_ERR_ARGUMENT, "unknown binary op");
    if (row_op != CTB_MIN && row_op != CTB_MAX) return fail(CTB_ERR_ARGUMENT, "row_op must be CTB_MIN or CTB_MAX");
    const int dt = a->dtype;
    if (dt != CTB_FLOAT32 && dt != CTB_FLOAT64) return fail(CTB_ERR_DTYPE, "fused rows take float32/float64");
    if (b->dtype != dt || c->dtype != dt || (y && y->dtype != dt))
        return fail(CTB_ERR_DTYPE, "fused rows take operands of one dtype");
    if (idx && idx->dtype != CTB_INT64) return fail(CTB_ERR_DTYPE, "row indices must be int64");
    if (a->ndim != 2 || a->strides[1] != 1 || a->shape[0] < 0 || a->shape[1] < 1)
        return fail(CTB_ERR_SHAPE, "a must be a 2-D [rows, cols] view with unit inner stride and cols >= 1");
    const int64_t R = a->shape[0], C = a->shape[1];
    if (C >= (int64_t(1) << 31)) return fail(CTB_ERR_SHAPE, "rows of 2^31 or more columns are not supported");
    auto row_operand = [&](const ctb_view* v, int& bcast) -> bool {
        int64_t n = 1;
        for (int d = 0; d < v->ndim; ++d) n *= v->shape[d];
        if (n == 1) {
            bcast = 1;
            return true;
        }
        bcast = 0;
        if (n != C) return false;
        // [C] or [1, C] with unit stride on the C dim
        for (int d = 0; d < v->ndim; ++d)
            if (v->shape[d] == C && v->strides[d] != 1) return false;
        return true;
    };
    if (!row_operand(b, p.b_bcast) || !row_operand(c, p.c_bcast))
        return fail(CTB_ERR_SHAPE, "b and c must be one contiguous row of `cols` elements, or scalars");
    if (y && (y->ndim != 2 || y->shape[0] != R || y->shape[1] != C || y->strides[1] != 1))
        return fail(CTB_ERR_SHAPE, "y must be a [rows, cols] view with unit inner stride");
    if (idx && !((idx->ndim == 1 && idx->shape[0] == R) || (idx->ndim == 2 && idx->shape[0] == R && idx->shape[1] == 1)))
        return fail(CTB_ERR_SHAPE, "row indices must be [rows] or [rows, 1]");
    p.a = a->data;
    p.b = b->data;
    p.c = c->data;
    p.y = y ? y->data : nullptr;
    p.idx = idx ? static_cast<int64_t*>(idx->data) : nullptr;
    p.rows = R;
    p.cols = C;
    p.a_row_stride = a->strides[0];
    p.y_row_stride = y ? y->strides[0] : 0;
    p.idx_stride = idx ? idx->strides[0] : 0;
    p.c_is_b = (c->data == b->data && p.c_bcast == p.b_bcast) ? 1 : 0;
    p.is_max = row_op == CTB_MAX;
    const int es = static_cast<int>(dtype_size(dt));
    vec = aligned16(a->data) && (!y || aligned16(y->data)) && (p.b_bcast || aligned16(b->data)) &&
          (p.c_bcast || aligned16(c->data)) && (p.a_row_stride * es) % 16 == 0 &&
          (!y || (p.y_row_stride * es) % 16 == 0);
    const size_t row_bytes = static_cast<size_t>((C * es + 15) / 16 * 16);
    smem = (p.c_is_b ? 1 : 2) * row_bytes;
    stage = smem <= kMaxStageBytes;
    if (!stage) smem = 0;
    // The pipelined loop (the chain alone, rows of a whole batch or more: 32 lanes x 4 packs,
    // 2 KiB) runs at exactly two CTAs per SM. Each kernel is a programmatic dependent of the one
    // before, so its CTAs are placed as SMs free up: with room for a third CTA on an SM, some SMs
    // took three and others one, and the slowest CTAs finished ~800 us after the fastest. Asking
    // for at least kPipeSmemBytes of shared memory leaves room for two on every SM.
    const bool whole_batch = !red && vec && C * es >= 32 * 4 * 16;
    if (stage && whole_batch && smem < kPipeSmemBytes) smem = kPipeSmemBytes;
    if (!red && !(vec && stage)) return -1;  // the chain-only kernel needs both
    const void* fn = nullptr;
    if (dt == CTB_FLOAT32) launch_ops<float>(op1, op2, vec, stage, red, 0, smem, p, nullptr, &fn);
    else launch_ops<double>(op1, op2, vec, stage, red, 0, smem, p, nullptr, &fn);
    if (smem > 48 * 1024) {
        if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
            return check_launch("fused rows smem attribute");
    }
    // One wave of warps, each taking rows warp, warp + nwarps, ...: as many rounds as a full wave
    // needs, and just enough warps for those rounds, so that the last round is as full as the
    // others (32768 rows over a full wave of 5920 warps would leave the sixth round 53% full;
    // 5464 warps keep it 99.7% full). The chain alone on rows of a whole batch or more (32 lanes
    // x 4 packs: 2 KiB) runs the pipelined loop at two CTAs (16 warps) per SM, where its loads in
    // flight match what the HBM serves best; in standalone kernels of the same loop on
    // [262144, 8192] float32, 24 warps per SM took 2788 us against 2596 us and 8 warps 3352 us.
    const int resident = resident_ctas(fn, 256, smem);
    const int64_t per_sm = whole_batch && resident > 2 ? 2 : resident;
    const int64_t wave = static_cast<int64_t>(sm_count()) * per_sm * 8;
    const int64_t rounds = R < 1 ? 1 : (R + wave - 1) / wave;
    const int64_t warps = (R + rounds - 1) / rounds;
    const int64_t ctas = (warps + 7) / 8;
    grid = static_cast<unsigned>(ctas < 1 ? 1 : ctas);
    return CTB_OK;
}

size_t fused_rows_scratch(int op1, int op2, const ctb_view* a, const ctb_view* b, const ctb_view* c,
                          const ctb_view* y, int row_op, const ctb_view* idx) {
    FusedRowsArgs p{};
    bool vec, stage;
    size_t smem;
    unsigned grid;
    if (plan_fused(op1, op2, a, b, c, y, row_op, idx, p, vec, stage, smem, grid)) return 0;
    return static_cast<size_t>(grid) * sizeof(double);
}

int fused_rows(int op1, int op2, const ctb_view* a, const ctb_view* b, const ctb_view* c,
               const ctb_view* y, int row_op, const ctb_view* idx, double* d_sum, void* scratch,
               size_t scratch_bytes, cudaStream_t st) {
    FusedRowsArgs p{};
    bool vec, stage;
    size_t smem;
    unsigned grid;
    if (int rc = plan_fused(op1, op2, a, b, c, y, row_op, idx, p, vec, stage, smem, grid)) return rc;
    if (d_sum) {
        const size_t need = static_cast<size_t>(grid) * sizeof(double);
        if (!scratch || scratch_bytes < need)
            return fail(CTB_ERR_SCRATCH, "scratch buffer too small: need " + std::to_string(need) + " bytes");
        p.partials = static_cast<double*>(scratch);
    }
    if (p.rows == 0) {
        if (d_sum && cudaMemsetAsync(d_sum, 0, sizeof(double), st) != cudaSuccess)
            return check_launch("fused rows");
        return CTB_OK;
    }
    if (a->dtype == CTB_FLOAT32) launch_ops<float>(op1, op2, vec, stage, true, grid, smem, p, st, nullptr);
    else launch_ops<double>(op1, op2, vec, stage, true, grid, smem, p, st, nullptr);
    int launches = 1;
    if (d_sum) {
        launch_dependent(fused_rows_combine, 1, 256, 0, st, p.partials, static_cast<int>(grid), d_sum);
        ++launches;
    }
    count_launch(launches);
    return check_launch("fused rows");
}

// Cross-GPU form: the launch above with the per-CTA partials in this rank's workspace and the
// last-CTA epilogue enabled (see the file comment). Every rank must make the same calls with the
// same epochs, in the same order.
int fused_rows_allsum(int op1, int op2, const ctb_view* a, const ctb_view* b, const ctb_view* c,
                      const ctb_view* y, int row_op, const ctb_view* idx, PeerWorkspace* const* d_peers,
                      int rank, int world, uint64_t epoch, const ctb_view* out_sum, double* d_parts,
                      uint64_t timeout_ns, unsigned long long* timeouts, PeerWorkspace* my_ws, cudaStream_t st) {
    FusedRowsArgs p{};
    bool vec, stage;
    size_t smem;
    unsigned grid;
    if (int rc = plan_fused(op1, op2, a, b, c, y, row_op, idx, p, vec, stage, smem, grid)) return rc;
    if (grid > static_cast<unsigned>(kPeerMaxCtas)) grid = kPeerMaxCtas;
    p.partials = my_ws->partials;
    p.peers = d_peers;
    p.rank = rank;
    p.world = world;
    p.epoch = epoch;
    p.timeout_ns = timeout_ns;
    p.out_sum = out_sum->data;
    p.out_sum_dtype = out_sum->dtype;
    p.out_parts = d_parts;
    p.timeouts = timeouts;
    // with no rows every CTA still runs the epilogue path (the grid is at least one CTA)
    if (a->dtype == CTB_FLOAT32) launch_ops<float>(op1, op2, vec, stage, true, grid, smem, p, st, nullptr);
    else launch_ops<double>(op1, op2, vec, stage, true, grid, smem, p, st, nullptr);
    count_launch();
    return check_launch("fused rows (cross-GPU sum)");
}

// ctb_binary_chain when the operands are rows of a [rows, cols] matrix and b, c are rows broadcast
// over it (or scalars): the row kernel above without its reductions. One warp per row with b and c
// in shared memory keeps more rows' loads in flight per SM than the elementwise row tiles, whose
// per-thread broadcast-row packs take registers. Measured against those tiles on B200, it is
// 1.5-7% faster on rows of 32 KiB or more (8192+ float32, 4096+ float64 columns) and 2-4% slower
// on rows of 4-16 KiB, so it takes rows of at least kChainRowBytesMin bytes (up to the staging
// limit), and at least kChainRowsMin of them, so that a one-wave grid of warps has rows to spare.
// Returns -1 (nothing launched) when the layout does not fit; the caller then plans the chain as
// any elementwise op.
constexpr int64_t kChainRowsMin = 16384;
constexpr int64_t kChainRowBytesMin = 32 * 1024;

int fused_chain_rows(int op1, int op2, const ctb_view* a, const ctb_view* b, const ctb_view* c,
                     const ctb_view* out, cudaStream_t st) {
    const int nd = out->ndim;
    if (nd < 1 || a->ndim != nd || a->dtype != out->dtype || b->dtype != out->dtype || c->dtype != out->dtype)
        return -1;
    const int64_t C = out->shape[nd - 1];
    int64_t n = 1;
    for (int d = 0; d < nd; ++d) n *= out->shape[d];
    if (C * static_cast<int64_t>(dtype_size(out->dtype)) < kChainRowBytesMin || n == 0) return -1;
    const int64_t R = n / C;
    if (R < kChainRowsMin) return -1;
    // a and out: the same shape, both contiguous row-major
    int64_t expect = 1;
    for (int d = nd - 1; d >= 0; --d) {
        if (a->shape[d] != out->shape[d]) return -1;
        if (out->shape[d] != 1 && (out->strides[d] != expect || a->strides[d] != expect)) return -1;
        expect *= out->shape[d];
    }
    // b, c: one element, or one unit-stride row of C broadcast over every other dim
    auto row_like = [&](const ctb_view* v) {
        if (v->ndim > nd) return false;
        int64_t m = 1;
        for (int d = 0; d < v->ndim; ++d) m *= v->shape[d];
        if (m == 1) return true;
        for (int d = 0; d < v->ndim - 1; ++d)
            if (v->shape[d] != 1) return false;
        return v->ndim >= 1 && v->shape[v->ndim - 1] == C && v->strides[v->ndim - 1] == 1;
    };
    if (!row_like(b) || !row_like(c)) return -1;
    ctb_view a2 = *a, y2 = *out;
    a2.ndim = y2.ndim = 2;
    a2.shape[0] = y2.shape[0] = R;
    a2.shape[1] = y2.shape[1] = C;
    a2.strides[0] = y2.strides[0] = C;
    a2.strides[1] = y2.strides[1] = 1;
    FusedRowsArgs p{};
    bool vec, stage;
    size_t smem;
    unsigned grid;
    const int rc = plan_fused(op1, op2, &a2, b, c, &y2, CTB_MIN, nullptr, p, vec, stage, smem, grid, false);
    if (rc) return rc;  // -1: unaligned, or rows too long to stage
    if (out->dtype == CTB_FLOAT32) launch_ops<float>(op1, op2, true, true, false, grid, smem, p, st, nullptr);
    else launch_ops<double>(op1, op2, true, true, false, grid, smem, p, st, nullptr);
    count_launch();
    return check_launch("chain rows");
}

}  // namespace ctb
