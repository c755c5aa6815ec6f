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
// address. Every call that needs scratch looks up the array's address on the current device with
// cudaGetSymbolAddress (cheap once the module is loaded; the first call on a device loads it, so
// make that first call before any stream capture). Nothing is cached, so the address stays right
// after a device reset or a new primary context.
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

// Device address of g_reduce_scratch in the current device's context.
int scratch_address(void** out) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_reduce_scratch);
    if (e != cudaSuccess || p == nullptr) {
        cudaGetLastError();
        return fail(CTB_ERR_CUDA, std::string("ctb_reduce_noalloc: cudaGetSymbolAddress failed: ") +
                                      cudaGetErrorString(e));
    }
    *out = p;
    return CTB_OK;
}

}  // namespace

size_t reduce_noalloc_capacity() { return kNoAllocScratchBytes; }

// The size check of ctb_reduce_noalloc: CTB_OK when `need` bytes fit the fixed array.
int noalloc_fits(size_t need) {
    if (need <= kNoAllocScratchBytes) return CTB_OK;
    return fail(CTB_ERR_SCRATCH, "ctb_reduce_noalloc: this reduction needs " + std::to_string(need) +
                                     " bytes of scratch, more than the fixed " +
                                     std::to_string(kNoAllocScratchBytes) +
                                     " bytes; use ctb_reduce with caller-provided scratch");
}

// Same validation and plan as ctb_reduce (the caller checks dtypes), then the launch with the
// static array as scratch. Split reductions write every partial slot before reading it, so the
// array needs no clearing between calls.
int reduce_noalloc(int op, const ctb_view* in, const ctb_view* out, uint32_t mask, cudaStream_t st) {
    size_t need = 0;
    const bool minmax = op == CTB_MAX || op == CTB_MIN;
    int rc = minmax ? minmax_dispatch(op, in, out, nullptr, mask, nullptr, 0, nullptr, &need)
                    : sum_like_dispatch(op, in, out, mask, nullptr, 0, nullptr, &need);
    if (rc) return rc;
    if ((rc = noalloc_fits(need))) return rc;
    void* scratch = nullptr;
    if (need > 0) {
        rc = scratch_address(&scratch);
        if (rc) return rc;
    }
    return minmax ? minmax_dispatch(op, in, out, nullptr, mask, scratch, kNoAllocScratchBytes, st, nullptr)
                  : sum_like_dispatch(op, in, out, mask, scratch, kNoAllocScratchBytes, st, nullptr);
}

}  // namespace ctb

extern "C" CTB_API int ctb_debug_noalloc_fits(size_t need) { return ctb::noalloc_fits(need); }
