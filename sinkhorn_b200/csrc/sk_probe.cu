// sk_probe.cu -- diagnostics with no reference counterpart:
//   * the device's ex2.approx throughput, the second floor of the Sinkhorn
//     roofline (every element of C costs one exponential per pass), measured
//     live next to the HBM figure instead of assumed;
//   * the bounded waits the pipelined kernels rely on (a local mbarrier, a
//     peer CTA's st.async into a cluster mbarrier, a grid barrier), run with
//     a short poll limit against a partner that does or does not arrive, so
//     a test can show that a wait whose partner never comes gives up,
//     reports SK_ERR_TIMEOUT and leaves the context usable.
#include "sk_cluster.cuh"
#include "sk_grid.cuh"
#include "sk_internal.h"

namespace sk {

constexpr int kProbeThreads = 256;
constexpr int kProbeChains = 8;  // independent ex2 chains per thread

__global__ void __launch_bounds__(kProbeThreads) k_probe_ex2(float* out, int rounds) {
    float v[kProbeChains];
#pragma unroll
    for (int c = 0; c < kProbeChains; ++c) v[c] = -1e-3f * (float)(threadIdx.x + c);
    for (int r = 0; r < rounds; ++r) {
#pragma unroll
        for (int c = 0; c < kProbeChains; ++c) {
            float y;
            asm volatile("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(v[c]));
            v[c] = y - 1.0f;  // stays in (-1, 0]: no overflow, no subnormals
        }
    }
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < kProbeChains; ++c) s += v[c];
    out[blockIdx.x * kProbeThreads + threadIdx.x] = s;  // keeps the chains live
}

// ---------------------------------------------------------------------------
// Bounded-wait probes. st: [0] error (2: a wait gave up, 3: wrong data),
// [4..7] a GridBarrier; zeroed by the host before each launch.

__global__ void k_probe_wait_mbar(int partner, uint32_t polls, unsigned* st) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 2);  // two arrivals complete the phase
        mbar_init_fence();
    }
    __syncthreads();
    if (threadIdx.x == 32 && partner) mbar_arrive(&bar);
    if (threadIdx.x == 0) {
        mbar_arrive(&bar);
        if (!mbar_wait(&bar, 0u, polls)) atomicMax(&st[0], 2u);
    }
    __syncthreads();
}

__global__ void __cluster_dims__(2, 1, 1) k_probe_wait_peer(int partner, uint32_t polls,
                                                            unsigned* st) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ __align__(8) float2 slot;
    __shared__ volatile int ab;
    const uint32_t rank = cluster_ctarank();
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        slot = make_float2(0.f, 0.f);
        ab = 0;
        mbar_init_fence();
    }
    __syncthreads();
    cluster_barrier();  // both CTAs' barriers exist before any remote arrival
    if (threadIdx.x == 0) {
        if (rank == 0) {
            // this CTA's arrival; the phase also waits for the peer's 8 bytes
            mbar_expect_tx(&bar, (uint32_t)sizeof(float2));
            if (!wait_peer(&bar, 0u, &ab, polls)) atomicMax(&st[0], 2u);
            else if (slot.x != 1.f || slot.y != 2.f) atomicMax(&st[0], 3u);
        } else if (partner) {
            st_async_f32x2(map_to_rank(&slot, 0), 1.f, 2.f, map_to_rank(&bar, 0));
        }
    }
    __syncthreads();
    cluster_barrier();  // neither CTA leaves while the other may touch its shared memory
}

__global__ void k_probe_wait_grid(int partner, uint32_t polls, unsigned* st) {
    __shared__ int ok;
    if (blockIdx.x == 1 && !partner) return;  // the partner never arrives
    if (!grid_barrier_bounded(reinterpret_cast<GridBarrier*>(st + 4), gridDim.x, polls, &ok) &&
        threadIdx.x == 0)
        atomicMax(&st[0], 2u);
}

}  // namespace sk

using namespace sk;

extern "C" {

size_t sk_probe_ex2_scratch_bytes(void) {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return sizeof(float) * (size_t)sms * 8 * kProbeThreads;
}

int sk_probe_ex2_rate(float* scratch, size_t scratch_bytes, double* ex2_per_second,
                      void* stream) {
    if (!ex2_per_second || !scratch) return fail(SK_ERR_ARG, "NULL argument");
    cudaStream_t s = (cudaStream_t)stream;
    int dev = 0, sms = 0;
    SK_CUDA(cudaGetDevice(&dev));
    SK_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int blocks = sms * 8;  // 8 CTAs of 256 threads per SM: every issue slot busy
    if (scratch_bytes < sizeof(float) * (size_t)blocks * kProbeThreads)
        return fail(SK_ERR_WORKSPACE, "scratch smaller than sk_probe_ex2_scratch_bytes");
    const int rounds = 4096;
    cudaEvent_t e0, e1;
    SK_CUDA(cudaEventCreate(&e0));
    SK_CUDA(cudaEventCreate(&e1));
    k_probe_ex2<<<blocks, kProbeThreads, 0, s>>>(scratch, rounds);  // warm-up
    SK_CUDA(cudaEventRecord(e0, s));
    k_probe_ex2<<<blocks, kProbeThreads, 0, s>>>(scratch, rounds);
    SK_CUDA(cudaEventRecord(e1, s));
    SK_LAUNCHED("k_probe_ex2 launch");
    SK_CUDA(cudaEventSynchronize(e1));
    float ms = 0.f;
    SK_CUDA(cudaEventElapsedTime(&ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    const double n = (double)blocks * kProbeThreads * (double)rounds * kProbeChains;
    *ex2_per_second = ms > 0.f ? n / ((double)ms * 1e-3) : 0.0;
    return SK_OK;
}

size_t sk_probe_wait_scratch_bytes(void) { return 8 * sizeof(unsigned); }

int sk_probe_wait_timeout(int kind, int partner, unsigned polls, void* scratch,
                          size_t scratch_bytes, void* stream) {
    clear_error();
    if (!scratch || scratch_bytes < sk_probe_wait_scratch_bytes())
        return fail(SK_ERR_WORKSPACE, "scratch smaller than sk_probe_wait_scratch_bytes");
    if (kind < 0 || kind > 2 || polls == 0u)
        return fail(SK_ERR_ARG, "kind must be 0 (mbarrier), 1 (cluster peer) or 2 (grid) "
                                "and polls positive");
    cudaStream_t s = (cudaStream_t)stream;
    unsigned* st = (unsigned*)scratch;
    const int p = partner ? 1 : 0;
    SK_CUDA(cudaMemsetAsync(st, 0, sk_probe_wait_scratch_bytes(), s));
    if (kind == 0) {
        k_probe_wait_mbar<<<1, 64, 0, s>>>(p, polls, st);
    } else if (kind == 1) {
        k_probe_wait_peer<<<2, 32, 0, s>>>(p, polls, st);
    } else {
        // both CTAs resident at once (the partner case waits for the other)
        void* args[] = {(void*)&p, (void*)&polls, (void*)&st};
        SK_CUDA(cudaLaunchCooperativeKernel((const void*)k_probe_wait_grid, dim3(2), dim3(32),
                                            args, 0, s));
    }
    SK_LAUNCHED("k_probe_wait launch");
    unsigned err = 0;
    SK_CUDA(cudaMemcpyAsync(&err, st, sizeof(unsigned), cudaMemcpyDeviceToHost, s));
    SK_CUDA(cudaStreamSynchronize(s));
    if (err == 2u) return fail(SK_ERR_TIMEOUT, "a bounded wait gave up: its partner never arrived");
    if (err) return fail(SK_ERR_DEVICE, "the probe's wait completed with the wrong data");
    return SK_OK;
}

}  // extern "C"
