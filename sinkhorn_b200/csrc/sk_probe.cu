// sk_probe.cu -- a diagnostic with no reference counterpart: the device's
// ex2.approx throughput, the second floor of the Sinkhorn roofline (every
// element of C costs one exponential per pass), measured live next to the
// HBM figure instead of assumed.
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

}  // extern "C"
