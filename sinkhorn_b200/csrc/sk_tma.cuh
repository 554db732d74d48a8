// sk_tma.cuh -- bulk asynchronous copies into shared memory and mbarriers
// (sm_90+ PTX, used on sm_100a), with bounded waits.
//
// A producer thread issues cp.async.bulk copies (global -> shared, completing
// a transaction count on an mbarrier); consumers wait on the mbarrier's phase
// parity. Every wait here gives up after a bounded number of polls and
// reports it, so a lost completion can never hang the GPU: the caller sets an
// error flag, lets its own copies land (again bounded) and returns.
// Every copy reads this GPU's own memory into the issuing CTA only.
#pragma once

#include <cuda.h>  // CUtensorMap (the type only; no driver-API linkage)
#include <stdint.h>

namespace sk {

// try_wait suspends for a hardware-chosen interval per poll; 1<<22 polls is
// far beyond any healthy wait (seconds) and still ends.
constexpr uint32_t kWaitPolls = 1u << 22;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

// make barrier initialisation visible to the async (bulk-copy) proxy
__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

// Raise the phase's expected transaction bytes without arriving (the arrive
// comes later, after the copies are issued and plain shared stores are made).
__device__ __forceinline__ void mbar_expect_tx_only(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          uint32_t polls = kWaitPolls) {
    for (uint32_t i = 0; i < polls; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

// bytes (multiple of 16, 16-byte aligned ends) from global to this CTA's
// shared memory; completion is counted on `bar` as transaction bytes.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
        "[%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// One tiled tensor copy global -> this CTA's shared memory: the box of the
// tensor map at coordinates (x, y, z) (x innermost; x * 4 bytes must be a
// multiple of 16). Rows / columns outside the tensor arrive as zeros; the
// transaction always counts the full box.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y,
                                            int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

}  // namespace sk
