// sk_cluster.cuh -- thread-block-cluster primitives (sm_90+ PTX, used on
// sm_100a) and bounded waits on them.
//
// The kernels that split a row of C over the CTAs of a cluster exchange small
// per-row results through distributed shared memory: st.async into a peer
// CTA's shared memory, completing transaction bytes on the peer's mbarrier,
// and an acquire.cluster try_wait on the receiving side. Every wait gives up
// after a bounded number of polls (or when an abort flag is raised), so a
// peer that never delivers cannot hang the GPU: the caller records an error
// and leaves through the cluster's final barrier.
// All traffic stays inside one cluster on one GPU.
#pragma once

#include <stdint.h>

#include "sk_tma.cuh"

namespace sk {

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Shared-memory address of `p` in the CTA of the cluster with the given rank.
__device__ __forceinline__ uint32_t map_to_rank(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}

// Asynchronous store of two floats into a peer CTA's shared memory that
// completes 8 transaction bytes on the peer's mbarrier (no fence: the data is
// visible to a thread that observes that barrier's phase complete).
__device__ __forceinline__ void st_async_f32x2(uint32_t addr, float x, float y, uint32_t bar) {
    asm volatile(
        "st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(
            addr),
        "f"(x), "f"(y), "r"(bar)
        : "memory");
}

// Plain 32-bit store into a peer CTA's shared memory (abort flags).
__device__ __forceinline__ void st_cluster_u32(uint32_t addr, uint32_t v) {
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Non-.aligned forms throughout: threads of a warp may arrive separately.
__device__ __forceinline__ void cluster_barrier() {
    asm volatile("barrier.cluster.arrive.release;\n\t"
                 "barrier.cluster.wait.acquire;" ::: "memory");
}

// Bounded wait for a local mbarrier phase; false on timeout or when the
// abort flag is raised.
__device__ __forceinline__ bool wait_full(uint64_t* bar, uint32_t parity, volatile int* ab,
                                          uint32_t polls = kWaitPolls) {
    for (uint32_t i = 0; i < polls; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*ab) return false;
    }
    return false;
}

// The same for a phase completed by peers of the cluster (acquire.cluster).
__device__ __forceinline__ bool wait_peer(uint64_t* bar, uint32_t parity, volatile int* ab,
                                          uint32_t polls = kWaitPolls) {
    for (uint32_t i = 0; i < polls; ++i) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if (*ab) return false;
    }
    return false;
}

// Warp-uniform forms: every lane polls (so each lane acquires the phase),
// and the warp agrees on the outcome, so a loop exit never splits a warp.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* ab) {
    return __all_sync(0xffffffffu, wait_full(bar, parity, ab));
}

__device__ __forceinline__ bool warp_wait_peer(uint64_t* bar, uint32_t parity, volatile int* ab) {
    return __all_sync(0xffffffffu, wait_peer(bar, parity, ab));
}

}  // namespace sk
