// common.cuh — shared device/host helpers for the sm_100a kernels behind include/ctb/ctb.h.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <string>
#include <type_traits>

#include "ctb/ctb.h"

namespace ctb {

constexpr int kMaxDims = CTB_MAX_DIMS;

// ------------------------------------------------------------------------------------------------
// errors and bookkeeping (capi.cu)

int fail(int status, const std::string& msg);         // records msg for ctb_last_error, returns status
int check_launch(const char* what);                   // cudaGetLastError -> CTB_ERR_CUDA
void count_launch(int n = 1);                         // feeds ctb_launch_count
int sm_count();                                       // SMs of the current device (cached)
// Resident CTAs per SM for `fn` at this block size / dynamic smem on the current device (cached;
// 4 when no device is present, e.g. when planning on a host without a GPU).
int resident_ctas(const void* fn, int block, size_t smem = 0);
size_t dtype_size(int dt);
int promote(int a, int b);                            // -1 for unsupported
const char* dtype_name(int dt);

// ------------------------------------------------------------------------------------------------
// 64-bit division by a runtime-invariant divisor: q = (umulhi(n, m) + n) >> s, valid for n < 2^63
// (round-up multiplier of Granlund & Montgomery, "Division by Invariant Integers using
// Multiplication", PLDI 1994, section 4). Host code builds it; kernels use it to decode linear
// indices into coordinates without a 64-bit divide.

struct FastDiv {
    uint64_t d = 1;
    uint64_t m = 0;
    uint32_t s = 0;

    FastDiv() = default;
    explicit FastDiv(uint64_t divisor) : d(divisor ? divisor : 1) {
        if (d == 1) {
            m = 0;
            s = 0;
            return;
        }
        uint32_t l = 0;
        while (l < 64 && (uint64_t(1) << l) < d) ++l;  // l = ceil(log2 d), 1..63
        const unsigned __int128 one = 1;
        const unsigned __int128 num = (one << (64 + l)) - (static_cast<unsigned __int128>(d) << 64);
        m = static_cast<uint64_t>(num / d) + 1;
        s = l;
    }

    __host__ __device__ __forceinline__ uint64_t div(uint64_t n) const {
        if (d == 1) return n;
#if defined(__CUDA_ARCH__)
        const uint64_t hi = __umul64hi(n, m);
#else
        const uint64_t hi =
            static_cast<uint64_t>((static_cast<unsigned __int128>(n) * m) >> 64);
#endif
        return (hi + n) >> s;
    }
    __host__ __device__ __forceinline__ void divmod(uint64_t n, uint64_t& q, uint64_t& r) const {
        q = div(n);
        r = n - q * d;
    }
};

// ------------------------------------------------------------------------------------------------
// element types

template <int DT> struct TypeOf;
template <> struct TypeOf<CTB_FLOAT32> { using type = float; };
template <> struct TypeOf<CTB_FLOAT64> { using type = double; };
template <> struct TypeOf<CTB_INT32> { using type = int32_t; };
template <> struct TypeOf<CTB_INT64> { using type = int64_t; };
template <> struct TypeOf<CTB_BOOL> { using type = uint8_t; };

template <class T> constexpr bool is_float_v = std::is_floating_point_v<T>;

// static_cast semantics of ctorch's cast (src/ops/cast_cpu.cpp:21-27); bool reads as 0/1.
template <class D, class S> __device__ __forceinline__ D cvt(S x) {
    if constexpr (std::is_same_v<S, uint8_t> && !std::is_same_v<D, uint8_t>) {
        return x ? D(1) : D(0);
    } else {
        return static_cast<D>(x);
    }
}

// Binary functors. Float ops use the round-to-nearest intrinsics so that no mul+add pair is ever
// contracted into an FMA (results must equal the separately-rounded CPU operations). Signed
// integers wrap through their unsigned representation (src/ops/functors.h:39-66).
// "No second op": the fused row kernel computes op1(x, b) alone (ctb_binary on row-broadcast rows).
constexpr int kOpNone = -1;

template <int OP> struct BinOp;
template <> struct BinOp<CTB_ADD> {
    template <class T> __device__ __forceinline__ static T apply(T a, T b) {
        if constexpr (std::is_same_v<T, float>) return __fadd_rn(a, b);
        else if constexpr (std::is_same_v<T, double>) return __dadd_rn(a, b);
        else return static_cast<T>(static_cast<std::make_unsigned_t<T>>(a) +
                                   static_cast<std::make_unsigned_t<T>>(b));
    }
};
template <> struct BinOp<CTB_SUB> {
    template <class T> __device__ __forceinline__ static T apply(T a, T b) {
        if constexpr (std::is_same_v<T, float>) return __fsub_rn(a, b);
        else if constexpr (std::is_same_v<T, double>) return __dsub_rn(a, b);
        else return static_cast<T>(static_cast<std::make_unsigned_t<T>>(a) -
                                   static_cast<std::make_unsigned_t<T>>(b));
    }
};
template <> struct BinOp<CTB_MUL> {
    template <class T> __device__ __forceinline__ static T apply(T a, T b) {
        if constexpr (std::is_same_v<T, float>) return __fmul_rn(a, b);
        else if constexpr (std::is_same_v<T, double>) return __dmul_rn(a, b);
        else return static_cast<T>(static_cast<std::make_unsigned_t<T>>(a) *
                                   static_cast<std::make_unsigned_t<T>>(b));
    }
};
template <> struct BinOp<CTB_DIV> {
    template <class T> __device__ __forceinline__ static T apply(T a, T b) {
        if constexpr (std::is_same_v<T, float>) return __fdiv_rn(a, b);
        else if constexpr (std::is_same_v<T, double>) return __ddiv_rn(a, b);
        else return a;  // integer division is refused on the host before any launch
    }
};

// ------------------------------------------------------------------------------------------------
// Vector access. A pack of N elements moves sizeof(T)*N bytes; packs of 16 bytes or more move as
// whole 16-byte chunks (a 32-byte pack that happens to start on a 32-byte boundary is stored in one
// piece, see store_pack), smaller packs as one naturally aligned access. The alignment rule is
// min(16, sizeof(T)*N) bytes at the start of every pack.

template <class T, int N> constexpr int pack_align() {
    return sizeof(T) * N >= 16 ? 16 : static_cast<int>(sizeof(T) * N);
}

template <class T, int N> struct alignas(pack_align<T, N>()) Pack {
    static_assert(sizeof(T) * N <= 16 || (sizeof(T) * N) % 16 == 0,
                  "packs above 16 bytes must be whole 16-byte chunks");
    T v[N];
};

template <class T, int N> __device__ __forceinline__ Pack<T, N> load_pack(const T* p) {
    Pack<T, N> r;
    if constexpr (sizeof(T) * N >= 16) {
        constexpr int kChunks = sizeof(T) * N / 16;
        const uint4* src = reinterpret_cast<const uint4*>(p);
        uint4* dst = reinterpret_cast<uint4*>(&r);
#pragma unroll
        for (int c = 0; c < kChunks; ++c) dst[c] = __ldg(src + c);
    } else {
        r = *reinterpret_cast<const Pack<T, N>*>(p);
    }
    return r;
}

// A pack of 16 bytes or more stored as 16-byte chunks, one store instruction each.
template <class T, int N> __device__ __forceinline__ void store_pack_split(T* p, const Pack<T, N>& v) {
    if constexpr (sizeof(T) * N >= 16) {
        constexpr int kChunks = sizeof(T) * N / 16;
        uint4* dst = reinterpret_cast<uint4*>(p);
        const uint4* src = reinterpret_cast<const uint4*>(&v);
#pragma unroll
        for (int c = 0; c < kChunks; ++c) dst[c] = src[c];
    } else {
        *reinterpret_cast<Pack<T, N>*>(p) = v;
    }
}

// A 32-byte pack on a 32-byte boundary is stored as one 32-byte-aligned object, which sm_100 can
// write with a single 256-bit store: each warp store is then one contiguous 1 KiB run instead of
// two instructions that each fill half of every sector. Measured on B200 with float64 outputs of
// float32 inputs (casts, adds and products with a broadcast operand): 11% faster. The per-row
// division paths keep store_pack_split, which measured 12% faster there.
struct alignas(32) Chunk32 {
    uint4 lo, hi;
};

template <class T, int N> __device__ __forceinline__ void store_pack(T* p, const Pack<T, N>& v) {
    if constexpr (sizeof(T) * N == 32) {
        if ((reinterpret_cast<uintptr_t>(p) & 31u) == 0) {
            Chunk32 c;
            c.lo = reinterpret_cast<const uint4*>(&v)[0];
            c.hi = reinterpret_cast<const uint4*>(&v)[1];
            *reinterpret_cast<Chunk32*>(p) = c;
            return;
        }
    }
    store_pack_split<T, N>(p, v);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <class A, class B> constexpr int max_size() { return sizeof(A) > sizeof(B) ? sizeof(A) : sizeof(B); }
template <class A, class B> constexpr int min_size() { return sizeof(A) < sizeof(B) ? sizeof(A) : sizeof(B); }

// Elements per thread-vector so that the narrowest participating type moves 16 bytes.
template <class O, class A, class B> constexpr int vec_elems() {
    constexpr int m = min_size<O, A>() < (int)sizeof(B) ? min_size<O, A>() : (int)sizeof(B);
    return 16 / m;
}

// ------------------------------------------------------------------------------------------------
// Programmatic dependent launch. Every kernel of this library is started with launch_dependent()
// and begins with dependent_wait(), before it touches memory: it may be scheduled while the kernel
// before it in the stream is still running (once every CTA of that kernel has called
// allow_dependents() or exited), its CTAs take SM room as it frees up, and they block in
// dependent_wait() until that kernel has completed and its writes are visible. Stream order is
// kept, and the launch and CTA start-up of each kernel overlap the previous one's tail: on B200,
// back-to-back [4096, 4096] float32 adds on the legacy stream take 24.0 us each this way against
// 25.7 us launched the ordinary way, the same as in a CUDA graph. Streaming kernels call
// allow_dependents() when their CTA's work is done, one-wave and small kernels at their start
// (their grid already holds the SMs, or needs few of them). A kernel started the ordinary way, or
// following a copy or another library's kernel, treats both instructions as no-ops.

__device__ __forceinline__ void allow_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void dependent_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <class... P, class... A>
cudaError_t launch_dependent(void (*kernel)(P...), unsigned grid, unsigned block, size_t smem,
                             cudaStream_t st, A... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<P>(args)...);
}

inline int ceil_div_int(int64_t a, int64_t b) { return static_cast<int>((a + b - 1) / b); }

// Grid size for a grid-stride kernel: enough CTAs to fill every SM `per_sm` times, never more
// than there is work for.
inline unsigned grid_for(int64_t work_items, int per_sm) {
    const int64_t cap = static_cast<int64_t>(sm_count()) * per_sm;
    int64_t g = work_items < cap ? work_items : cap;
    return static_cast<unsigned>(g < 1 ? 1 : g);
}

}  // namespace ctb
