// async_copy.cuh — bulk asynchronous copies (global -> shared) completed through mbarriers, the
// sm_100a way to keep many bytes in flight without holding them in registers.
//
// A stage ring works as follows. A producer warp waits for a stage to be free (its "empty"
// barrier), posts the bytes it is about to copy (arrive.expect_tx on the stage's "full" barrier)
// and issues copies that complete against that barrier: bulk copies (cp.async.bulk, one
// contiguous range each) or tensor copies (cp.async.bulk.tensor, one box of rows of a tensor
// described by a tensor map). Consumers wait on "full", read the stage from shared memory and
// arrive on "empty".
//
// Every wait here is bounded in time. A wait that runs out returns false; the kernel then counts
// the event in a device counter (its address comes in the kernel's arguments, read on the host
// with ctb_wait_timeouts), stops issuing work, lets the copies it has in flight land (again with
// a bound) and returns, leaving its outputs unwritten. No copy here uses cluster multicast: every
// source is this GPU's own global memory, read by the CTA that consumes it.
#pragma once

#include <cuda.h>  // CUtensorMap

#include <cstdint>

namespace ctb {

// How long one wait may take before the kernel gives up (about a second: a stage normally
// completes in microseconds).
constexpr uint64_t kWaitLimitNs = 1000000000ull;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t arrivals) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(arrivals) : "memory");
}

// Makes the barrier initialisation visible to the asynchronous (bulk copy) proxy.
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// One arrival plus `bytes` of expected transaction count: the phase completes once every arrival
// is in and that many bytes have landed.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

// True once the phase with the given parity has completed.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Waits for the phase of `parity` to complete, for at most `limit_ns`. Returns false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns = kWaitLimitNs) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
#pragma unroll 1
        for (int i = 0; i < 32; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (global_ns() - t0 > limit_ns) return false;
    }
}

// Copies `bytes` (a multiple of 16; both addresses 16-byte aligned) from this GPU's global memory
// into this CTA's shared memory; completion is counted on `bar`.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(smem_dst)),
        "l"(gsrc), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// Copies one box of a 3-D tensor (described by `map`, a __grid_constant__ kernel parameter) at
// element coordinates (x, y, z) into this CTA's shared memory, row after row; completion is
// counted on `bar`. x times the element size must be a multiple of 16 bytes; rows past the
// tensor's extent arrive as zeros. smem_dst is 128-byte aligned.
__device__ __forceinline__ void tensor_load_3d(void* smem_dst, const CUtensorMap* map, int x, int y, int z,
                                               uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_addr(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
        : "memory");
}

// Records a timed-out wait (the host reads the count with ctb_wait_timeouts).
__device__ __forceinline__ void note_timeout(unsigned long long* counter) {
    if (counter) atomicAdd(counter, 1ull);
}

}  // namespace ctb
