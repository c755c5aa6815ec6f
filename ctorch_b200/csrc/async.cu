// async.cu — the device counter of timed-out waits that the bulk-copy kernels report to
// (async_copy.cuh), its C-ABI reader, a self-test of the bounded wait, and the tensor maps of the
// strip column kernel.
#include <cudaTypedefs.h>

#include <mutex>
#include <string>

#include "async_copy.cuh"
#include "common.cuh"
#include "plan.cuh"

namespace ctb {

namespace {

__device__ unsigned long long g_wait_timeouts;

constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned long long* g_counter[kMaxDevices] = {};

// Waits on a barrier that nothing ever arrives at, for `limit_ns`, and records the outcome:
// result[0] = 1 if the wait (wrongly) completed, 0 if it timed out as it must.
__global__ void wait_self_test(uint64_t limit_ns, unsigned long long* counter, int* result) {
    __shared__ uint64_t bar;
    if (threadIdx.x != 0) return;
    mbar_init(&bar, 1);
    mbar_fence_init();
    const bool done = mbar_wait(&bar, 0u, limit_ns);
    if (!done) note_timeout(counter);
    result[0] = done ? 1 : 0;
}

}  // namespace

unsigned long long* wait_timeout_counter() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_counter[dev] == nullptr) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_wait_timeouts) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        g_counter[dev] = static_cast<unsigned long long*>(p);
    }
    return g_counter[dev];
}

namespace {

// The driver's tensor-map encoder, fetched once through the runtime (no link against libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            f = nullptr;
        }
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }();
    return fn;
}

}  // namespace

bool encode_strip_map(RedPlan& plan, int elem_bytes) {
    const RedArgs& a = plan.args;
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc || (elem_bytes != 4 && elem_bytes != 8) || a.strip_pk < 1) return false;
    const int64_t vec = 16 / elem_bytes;
    const int64_t batch = a.kept / a.N;
    const int64_t rows = static_cast<int64_t>(kColsConsumers / a.strip_pk) * kStripRows;
    const int64_t batch_stride = a.rank_k == 2 ? a.stride_k[0] : a.K * a.strideK;
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(a.N), static_cast<cuuint64_t>(a.K),
                                static_cast<cuuint64_t>(batch)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(a.strideK * elem_bytes),
                                   static_cast<cuuint64_t>(batch_stride * elem_bytes)};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(a.strip_pk * vec), static_cast<cuuint32_t>(rows), 1u};
    const cuuint32_t unit[3] = {1u, 1u, 1u};
    const CUresult r = enc(&plan.strip_map, elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_UINT32 : CU_TENSOR_MAP_DATA_TYPE_UINT64,
                           3, const_cast<void*>(a.in), dims, strides, box, unit, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace ctb

extern "C" {

CTB_API int ctb_wait_timeouts(uint64_t* count) {
    using namespace ctb;
    if (!count) return fail(CTB_ERR_ARGUMENT, "ctb_wait_timeouts: null count");
    unsigned long long* p = wait_timeout_counter();
    if (!p) return fail(CTB_ERR_CUDA, "ctb_wait_timeouts: device counter unavailable");
    unsigned long long v = 0;
    const cudaError_t e = cudaMemcpy(&v, p, sizeof(v), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(CTB_ERR_CUDA, std::string("ctb_wait_timeouts: ") + cudaGetErrorString(e));
    }
    *count = static_cast<uint64_t>(v);
    return CTB_OK;
}

CTB_API int ctb_debug_wait_timeout(uint64_t limit_ns, int* completed) {
    using namespace ctb;
    if (!completed) return fail(CTB_ERR_ARGUMENT, "ctb_debug_wait_timeout: null result");
    if (limit_ns > 100000000ull) return fail(CTB_ERR_ARGUMENT, "ctb_debug_wait_timeout: limit above 100 ms");
    unsigned long long* counter = wait_timeout_counter();
    if (!counter) return fail(CTB_ERR_CUDA, "ctb_debug_wait_timeout: device counter unavailable");
    int* d = nullptr;
    if (cudaMalloc(&d, sizeof(int)) != cudaSuccess) {
        cudaGetLastError();
        return fail(CTB_ERR_CUDA, "ctb_debug_wait_timeout: cudaMalloc failed");
    }
    wait_self_test<<<1, 32>>>(limit_ns, counter, d);
    int rc = check_launch("ctb_debug_wait_timeout");
    int h = -1;
    if (rc == CTB_OK) {
        const cudaError_t e = cudaMemcpy(&h, d, sizeof(int), cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) {
            cudaGetLastError();
            rc = fail(CTB_ERR_CUDA, std::string("ctb_debug_wait_timeout: ") + cudaGetErrorString(e));
        }
    }
    cudaFree(d);
    *completed = h;
    return rc;
}

}  // extern "C"
