// sk_noalloc.cu -- the column softmin without a caller-provided workspace.
//
// Who needs it: callers that cannot allocate device memory at the moment
// they call in. A host application whose memory manager reserved the GPU's
// memory for itself at start-up (frameworks that preallocate most of HBM)
// has nothing left to hand out; a latency-critical service may forbid
// cudaMalloc on its request path because an allocation can block and
// synchronise the device; and a foreign-language binding may have no device
// allocator at all. For them sk_lse_col_noalloc runs the same kernel as
// sk_lse_col, with its scratch (column-tile tickets and per-band partial
// LSEs) taken from a fixed array compiled into this library.
//
// Limits and sharing:
//   * the array holds kNoAllocScratchBytes (8 MiB); a problem whose scratch
//     (the size sk_lse_col_workspace_bytes reports) is larger is rejected
//     with SK_ERR_WORKSPACE before anything is launched;
//   * every GPU that loads the library keeps the 8 MiB until the process
//     exits;
//   * all calls on a device share the one array and it keeps the contents of
//     the last call: the tickets, which must start at zero, are cleared at the
//     start of every call, and the partials are always written before they
//     are read. Two calls that overlap on the GPU (e.g. on two streams at
//     once) race on the array -- order them on one stream or with events;
//   * the first call on each device looks up the array's device address
//     (cudaGetSymbolAddress, with that device current) and caches it; make
//     that first call before any stream capture. After cudaDeviceReset the
//     cached address is stale: do not call in again on that device in the
//     same process.
// Nothing here calls cudaMalloc, cudaFree or any other allocating routine.
#include <mutex>

#include "sk_internal.h"
#include "sk_solve.cuh"

namespace sk {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;

// Device scratch of sk_lse_col_noalloc. In host code this name is only a
// host-side stand-in for the symbol, never a usable device address: the
// address comes from cudaGetSymbolAddress (noalloc_scratch below).
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
static void* g_scratch_addr[kMaxDevices];
static std::mutex g_scratch_mu;

// Device address of g_noalloc_scratch on the current device (looked up once
// per device, with that device current).
static int noalloc_scratch(void** out) {
    int dev = -1;
    SK_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices)
        return fail(SK_ERR_ARG, "device ordinal out of range for the built-in scratch");
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (g_scratch_addr[dev] == nullptr) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(built-in scratch)");
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return SK_OK;
}

}  // namespace sk

using namespace sk;

extern "C" {

int sk_lse_col_noalloc(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                       int64_t sCn, int64_t sCm, const float* f, double epsilon, float* out,
                       void* stream) {
    clear_error();
    if (int e = check_problem(C, B, N, M, epsilon)) return e;
    if (!f || !out) return fail(SK_ERR_ARG, "f and out must be non-NULL");
    const size_t need = sk_lse_col_workspace_bytes(B, N, M);
    if (need > kNoAllocScratchBytes)
        return fail(SK_ERR_WORKSPACE,
                    "sk_lse_col_noalloc: this problem needs " + std::to_string(need) +
                        " bytes of scratch but the built-in scratch holds " +
                        std::to_string(kNoAllocScratchBytes) +
                        " bytes (8 MiB); call sk_lse_col with a workspace instead");
    void* ws = nullptr;
    if (int e = noalloc_scratch(&ws)) return e;
    cudaStream_t s = (cudaStream_t)stream;
    const SweepPlan p = make_plan(C, B, N, M, sCb, sCn, sCm);
    const size_t tick_bytes = sizeof(unsigned) * B * max_col_tiles(M);
    unsigned* tickets = (unsigned*)ws;
    float* partial = (float*)((char*)ws + align_up(tick_bytes));
    SK_CUDA(cudaMemsetAsync(tickets, 0, tick_bytes, s));
    ColArgs c{};
    c.C = C;
    c.sCb = sCb;
    c.sCn = sCn;
    c.sCm = sCm;
    c.B = B;
    c.N = N;
    c.M = M;
    c.f_eff = f;
    c.g_out = out;
    c.partial = partial;
    c.tickets = tickets;
    c.ntiles = p.ntiles;
    c.nbands = p.nbands;
    c.band_rows = p.band_rows;
    c.k = (float)(1.0 / epsilon);
    c.eps = (float)epsilon;
    c.plain = 1;
    launch_col(p, c, s);
    SK_LAUNCHED("k_col_sweep launch (built-in scratch)");
    return SK_OK;
}

}  // extern "C"
