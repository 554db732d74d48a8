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

// Barrier k (k = 1, 2, ...) of a launch on a monotonically increasing
// arrival counter that is zero when the launch starts and sits on a cache
// line of its own: every CTA adds 1 (a fire-and-forget reduction) and waits
// until the counter reaches k * nblocks (wrap-around compare). No reset and no
// second word, so an arrival costs one reduction and the waiters only read.
// One thread per CTA; `abort` is polled every 32 polls; returns false on abort
// or when the polls run out (the caller then raises the abort word).
__device__ __forceinline__ bool grid_sync_counter(unsigned* count, unsigned target,
                                                  const unsigned* abort, uint32_t polls) {
    __threadfence();  // this CTA's writes before its arrival
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(count) : "memory");
    for (uint32_t i = 0; i < polls; ++i) {
        if ((int)(ld_acquire_gpu(count) - target) >= 0) {
            __threadfence();  // the other CTAs' writes after the barrier
            return true;
        }
        if ((i & 31u) == 31u && ld_acquire_gpu(abort) != 0u) return false;
        __nanosleep(20);
    }
    return false;
}

// Release store / acquire load at system scope: the flags another GPU reads
// or writes through peer memory (sk_peer.cu).
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Bounded wait (thread 0 of the calling CTA) until every flag holds at least
// `seq`; false when the polls run out (a rank that never delivers).
__device__ __forceinline__ bool peer_wait_flags(const unsigned* flags, int P, unsigned seq) {
    for (uint32_t i = 0; i < (1u << 24); ++i) {  // with the sleep below: seconds, then give up
        bool all = true;
        for (int p = 0; p < P; ++p)
            if ((int)(ld_acquire_sys(flags + p) - seq) < 0) {
                all = false;
                break;
            }
        if (all) return true;
        __nanosleep(32);
    }
    return false;
}

// Named barrier of `nthreads` threads (whole warps) of the CTA.
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

}  // namespace sk
