// index_select.cu — gather along one dim (ctorch::index_select, src/ops/indexing_cpu.cpp:35-101).
//
// Two launches on the caller's stream, no host synchronisation in between:
//   1. idx_validate: every index checked against [-size, size) (before normalising, so INT64_MIN
//      is caught, src/ops/indexing_cpu.cpp:59-66); the first failure raises a device flag and
//      records the offending value.
//   2. the gather, which returns at once if the flag is up, so nothing is written on error.
// The row gather moves whole contiguous rows (the dims after `dim`) warp by warp in 16-byte (or
// the widest aligned) units, four rows in flight per warp; the index is read once per row. The
// general gather decodes each element. Element values are copied as raw bytes, so results are
// bit-exact for every dtype (ctorch's CUDA path is one thread per element,
// src/ops/indexing_cuda.cu:108-129).
#include "common.cuh"
#include "plan.cuh"

namespace ctb {

struct GatherArgs {
    const char* src;
    char* out;
    const void* idx;
    int32_t* status;     // [0] flag, bytes 8..15 offending value
    int64_t n_idx;
    int64_t idx_stride;  // elements
    int64_t dim_size;
    int64_t dim_stride;  // src elements
    int es;              // element bytes
    // row path
    int64_t row_bytes;   // L * es
    int64_t rows;        // outer * n_idx
    int rank_o;          // outer dims (before `dim`)
    int64_t stride_o[kMaxDims];  // src strides of the outer dims (elements)
    FastDiv div_o[kMaxDims];
    FastDiv div_n;       // n_idx
    // general path
    int rank, dim;
    int64_t n_out;
    int64_t src_stride[kMaxDims], out_stride[kMaxDims];
    FastDiv div[kMaxDims];
};

template <class I>
__global__ void idx_validate(const I* idx, int64_t n, int64_t stride, int64_t size, int32_t* status) {
    dependent_wait();  // the previous kernel in the stream has completed and its writes are visible
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nthr = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = tid; i < n; i += nthr) {
        const int64_t raw = static_cast<int64_t>(idx[i * stride]);
        if (raw < -size || raw >= size) {
            if (atomicCAS(reinterpret_cast<int*>(status), 0, 1) == 0)
                *reinterpret_cast<long long*>(status + 2) = raw;
        }
    }
    allow_dependents();  // the next kernel in the stream may launch while this one winds down
}

template <class I>
__device__ __forceinline__ int64_t resolve(const GatherArgs& p, int64_t j) {
    int64_t v = static_cast<int64_t>(static_cast<const I*>(p.idx)[j * p.idx_stride]);
    return v < 0 ? v + p.dim_size : v;
}

// Warp per output row; U rows in flight per warp; unit VB bytes.
template <class I, class VT>
__global__ void __launch_bounds__(256, 4) gather_rows(GatherArgs p) {
    dependent_wait();  // the previous kernel in the stream has completed and its writes are visible
    constexpr int U = 4;
    constexpr int VB = sizeof(VT);
    if (*reinterpret_cast<volatile int32_t*>(p.status) != 0) return;
    const int lane = threadIdx.x & 31;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    const int64_t units = p.row_bytes / VB;
    for (int64_t r0 = warp; r0 < p.rows; r0 += nwarps * U) {
        const VT* s[U];
        VT* d[U];
        bool ok[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t r = r0 + u * nwarps;
            ok[u] = r < p.rows;
            s[u] = nullptr;
            d[u] = nullptr;
            if (ok[u]) {
                uint64_t o, j;
                p.div_n.divmod(static_cast<uint64_t>(r), o, j);
                int64_t off = resolve<I>(p, static_cast<int64_t>(j)) * p.dim_stride;
                for (int dd = p.rank_o - 1; dd >= 0; --dd) {
                    uint64_t q, c;
                    p.div_o[dd].divmod(o, q, c);
                    off += static_cast<int64_t>(c) * p.stride_o[dd];
                    o = q;
                }
                s[u] = reinterpret_cast<const VT*>(p.src + off * p.es);
                d[u] = reinterpret_cast<VT*>(p.out + r * p.row_bytes);
            }
        }
        for (int64_t c0 = lane; c0 < units; c0 += 64) {
            VT x[U][2];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if (ok[u]) {
                    x[u][0] = s[u][c0];
                    if (c0 + 32 < units) x[u][1] = s[u][c0 + 32];
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if (ok[u]) {
                    d[u][c0] = x[u][0];
                    if (c0 + 32 < units) d[u][c0 + 32] = x[u][1];
                }
            }
        }
    }
    allow_dependents();  // the next kernel in the stream may launch while this one winds down
}

template <class I, class ET>
__global__ void __launch_bounds__(256) gather_general(GatherArgs p) {
    dependent_wait();  // the previous kernel in the stream has completed and its writes are visible
    if (*reinterpret_cast<volatile int32_t*>(p.status) != 0) return;
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nthr = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const ET* src = reinterpret_cast<const ET*>(p.src);
    ET* out = reinterpret_cast<ET*>(p.out);
    for (int64_t i = tid; i < p.n_out; i += nthr) {
        uint64_t rem = static_cast<uint64_t>(i);
        int64_t so = 0, oo = 0;
        for (int d = p.rank - 1; d >= 0; --d) {
            uint64_t q, c;
            p.div[d].divmod(rem, q, c);
            const int64_t ci = static_cast<int64_t>(c);
            so += (d == p.dim ? resolve<I>(p, ci) : ci) * p.src_stride[d];
            oo += ci * p.out_stride[d];
            rem = q;
        }
        out[oo] = src[so];
    }
    allow_dependents();  // the next kernel in the stream may launch while this one winds down
}

template <class I>
int gather_typed(const ctb_view* src, int dim, const ctb_view* idx, const ctb_view* out,
                 int32_t* status, cudaStream_t st) {
    GatherArgs p{};
    const int rank = src->ndim;
    const int es = static_cast<int>(dtype_size(src->dtype));
    p.src = static_cast<const char*>(src->data);
    p.out = static_cast<char*>(out->data);
    p.idx = idx->data;
    p.status = status;
    p.n_idx = idx->shape[0];
    p.idx_stride = idx->strides[0];
    p.dim_size = src->shape[dim];
    p.dim_stride = src->strides[dim];
    p.es = es;

    if (cudaMemsetAsync(status, 0, 16, st) != cudaSuccess) return check_launch("index_select status reset");
    if (p.n_idx == 0) return CTB_OK;
    {
        const int64_t blocks = (p.n_idx + 255) / 256;
        launch_dependent(idx_validate<I>, grid_for(blocks, 8), 256, 0, st, static_cast<const I*>(idx->data), p.n_idx,
                                                            p.idx_stride, p.dim_size, status);
        count_launch();
        const int rc = check_launch("index_select validate");
        if (rc) return rc;
    }
    int64_t n_out = 1;
    for (int d = 0; d < rank; ++d) n_out *= out->shape[d];
    if (n_out == 0) return CTB_OK;

    // Row path: out contiguous, src's dims after `dim` form one contiguous run.
    bool out_contig = true;
    {
        int64_t expect = 1;
        for (int d = rank - 1; d >= 0; --d) {
            if (out->shape[d] != 1 && out->strides[d] != expect) out_contig = false;
            expect *= out->shape[d];
        }
    }
    bool inner_contig = true;
    int64_t L = 1;
    for (int d = rank - 1; d > dim; --d) {
        if (src->shape[d] != 1 && src->strides[d] != L) inner_contig = false;
        L *= src->shape[d];
    }
    if (out_contig && inner_contig) {
        p.row_bytes = L * es;
        p.rank_o = 0;
        int64_t outer = 1;
        for (int d = 0; d < dim; ++d) {
            if (src->shape[d] == 1) continue;
            p.stride_o[p.rank_o] = src->strides[d];
            p.div_o[p.rank_o] = FastDiv(static_cast<uint64_t>(src->shape[d]));
            ++p.rank_o;
            outer *= src->shape[d];
        }
        p.rows = outer * p.n_idx;
        p.div_n = FastDiv(static_cast<uint64_t>(p.n_idx));
        // widest unit that keeps every row start aligned
        uint64_t g = static_cast<uint64_t>(p.row_bytes) | reinterpret_cast<uintptr_t>(p.src) |
                     reinterpret_cast<uintptr_t>(p.out) | static_cast<uint64_t>(p.dim_stride * es);
        for (int d = 0; d < p.rank_o; ++d) g |= static_cast<uint64_t>(p.stride_o[d] * es);
        const int64_t warps = p.rows;
        const unsigned grid = grid_for((warps + 7) / 8, 16);
        if ((g & 15u) == 0) launch_dependent(gather_rows<I, uint4>, grid, 256, 0, st, p);
        else if ((g & 7u) == 0) launch_dependent(gather_rows<I, uint2>, grid, 256, 0, st, p);
        else if ((g & 3u) == 0) launch_dependent(gather_rows<I, uint32_t>, grid, 256, 0, st, p);
        else if ((g & 1u) == 0) launch_dependent(gather_rows<I, uint16_t>, grid, 256, 0, st, p);
        else launch_dependent(gather_rows<I, uint8_t>, grid, 256, 0, st, p);
        count_launch();
        return check_launch("index_select gather");
    }
    p.rank = rank;
    p.dim = dim;
    p.n_out = n_out;
    for (int d = 0; d < rank; ++d) {
        p.src_stride[d] = src->strides[d];
        p.out_stride[d] = out->strides[d];
        p.div[d] = FastDiv(static_cast<uint64_t>(out->shape[d]));
    }
    const unsigned grid = grid_for((n_out + 255) / 256, 16);
    switch (es) {
    case 1: launch_dependent(gather_general<I, uint8_t>, grid, 256, 0, st, p); break;
    case 2: launch_dependent(gather_general<I, uint16_t>, grid, 256, 0, st, p); break;
    case 4: launch_dependent(gather_general<I, uint32_t>, grid, 256, 0, st, p); break;
    default: launch_dependent(gather_general<I, uint64_t>, grid, 256, 0, st, p); break;
    }
    count_launch();
    return check_launch("index_select gather");
}

// dtypes/shapes validated by the caller (capi.cu).
int index_select_dispatch(const ctb_view* src, int dim, const ctb_view* idx, const ctb_view* out,
                          int32_t* status, cudaStream_t st) {
    if (idx->dtype == CTB_INT32) return gather_typed<int32_t>(src, dim, idx, out, status, st);
    return gather_typed<int64_t>(src, dim, idx, out, status, st);
}

}  // namespace ctb
