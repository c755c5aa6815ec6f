// noalloc.cu — ctb_reduce_noalloc: the reductions of ctb_reduce with their scratch in a
// fixed-size array that lives in the library's device image, so the call allocates nothing.
//
// Who needs it: hosts that cannot hand the backend scratch memory. A plain C or FFI caller that
// owns no device allocator of its own has nothing to pass as `scratch`, and a process that fixes
// its device memory at start-up must not call cudaMalloc later (it can fail under fragmentation
// and it synchronises the device). ctb_reduce asks the caller for scratch; this entry point uses
// g_reduce_scratch below instead.
//
// The array is a file-scope __device__ variable, so host code cannot use its name as a device
// address. On the first call on each device (with that device current) the entry point looks up
// the array's device address with cudaGetSymbolAddress and caches it; make that first call before
// any stream capture. Every later call on the device reuses the same array.
#include <mutex>
#include <string>

#include "common.cuh"

namespace ctb {

int sum_like_dispatch(int op, const ctb_view* in, const ctb_view* out, uint32_t mask, void* scratch,
                      size_t sb, cudaStream_t st, size_t* need_only);
int minmax_dispatch(int op, const ctb_view* in, const ctb_view* values, const ctb_view* indices,
                    uint32_t mask, void* scratch, size_t sb, cudaStream_t st, size_t* need_only);

namespace {

// 4 MiB per device: enough for any split reduction whose outputs times splits times state size
// fits (a column max with indices over 8192 columns split 9 ways needs 1.2 MB).
constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;

__device__ __align__(256) unsigned char g_reduce_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_reduce_scratch on the current device, looked up once per device.
int scratch_address(void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return check_launch("ctb_reduce_noalloc: cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices)
        return fail(CTB_ERR_ARGUMENT, "ctb_reduce_noalloc: device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_scratch_ptr[dev] == nullptr) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_reduce_scratch);
        if (e != cudaSuccess || p == nullptr) {
            cudaGetLastError();
            return fail(CTB_ERR_CUDA, std::string("ctb_reduce_noalloc: cudaGetSymbolAddress failed: ") +
                                          cudaGetErrorString(e));
        }
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return CTB_OK;
}

}  // namespace

size_t reduce_noalloc_capacity() { return kNoAllocScratchBytes; }

// Same validation and plan as ctb_reduce (the caller checks dtypes), then the launch with the
// static array as scratch. Split reductions write every partial slot before reading it, so the
// array needs no clearing between calls.
int reduce_noalloc(int op, const ctb_view* in, const ctb_view* out, uint32_t mask, cudaStream_t st) {
    size_t need = 0;
    const bool minmax = op == CTB_MAX || op == CTB_MIN;
    int rc = minmax ? minmax_dispatch(op, in, out, nullptr, mask, nullptr, 0, nullptr, &need)
                    : sum_like_dispatch(op, in, out, mask, nullptr, 0, nullptr, &need);
    if (rc) return rc;
    if (need > kNoAllocScratchBytes)
        return fail(CTB_ERR_SCRATCH, "ctb_reduce_noalloc: this reduction needs " + std::to_string(need) +
                                         " bytes of scratch, more than the fixed " +
                                         std::to_string(kNoAllocScratchBytes) +
                                         " bytes; use ctb_reduce with caller-provided scratch");
    void* scratch = nullptr;
    if (need > 0) {
        rc = scratch_address(&scratch);
        if (rc) return rc;
    }
    return minmax ? minmax_dispatch(op, in, out, nullptr, mask, scratch, kNoAllocScratchBytes, st, nullptr)
                  : sum_like_dispatch(op, in, out, mask, scratch, kNoAllocScratchBytes, st, nullptr);
}

}  // namespace ctb
