// sk_grid.cuh -- a bounded barrier over all CTAs of a grid.
//
// For kernels whose CTAs are all resident at once (a cooperative launch, or
// a grid no larger than what the occupancy query reports for one wave): an
// arrival counter and a generation word in global memory, both zero before
// the first use. Thread 0 of each CTA arrives; the last arrival resets the
// counter and bumps the generation; the others poll the generation with
// short sleeps for a bounded number of polls. A waiter that gives up raises
// the shared abort word, which every other waiter polls too, so one lost CTA
// ends every wait quickly instead of each running out its own bound; after
// an abort the kernel must leave (the counter is no longer consistent).
#pragma once

#include <stdint.h>

namespace sk {

struct GridBarrier {
    unsigned count;  // arrivals of the current generation
    unsigned gen;    // generation, bumped by the last arrival
    unsigned abort;  // non-zero: a wait gave up (or the caller aborted)
    unsigned pad;
};

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Every thread of every CTA calls this. Returns false (uniformly within the
// CTA) when the barrier was aborted or a wait ran out of polls.
__device__ __forceinline__ bool grid_barrier_bounded(GridBarrier* gb, unsigned nblocks,
                                                     uint32_t polls, int* sh_ok) {
    __syncthreads();
    if (threadIdx.x == 0) {
        bool ok = ld_acquire_gpu(&gb->abort) == 0u;
        if (ok) {
            const unsigned g0 = ld_acquire_gpu(&gb->gen);
            __threadfence();  // this CTA's writes before its arrival
            if (atomicAdd(&gb->count, 1u) == nblocks - 1u) {
                atomicExch(&gb->count, 0u);
                __threadfence();
                atomicAdd(&gb->gen, 1u);
            } else {
                uint32_t i = 0;
                for (; i < polls; ++i) {
                    if (ld_acquire_gpu(&gb->gen) != g0) break;
                    if (ld_acquire_gpu(&gb->abort) != 0u) {
                        i = polls;
                        break;
                    }
                    __nanosleep(32);
                }
                if (i >= polls) {
                    ok = false;
                    atomicExch(&gb->abort, 1u);
                }
            }
            __threadfence();  // the other CTAs' writes after the barrier
        }
        *sh_ok = ok ? 1 : 0;
    }
    __syncthreads();
    return *sh_ok != 0;
}

}  // namespace sk
