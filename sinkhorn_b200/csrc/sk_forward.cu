// sk_forward.cu -- Sinkhorn forward solve and standalone softmins (C ABI).
//
// One iteration = one row sweep (f-update) + one column sweep (g-update with
// the band merge, residual and convergence decision fused into its last
// CTAs). The host only enqueues: convergence is decided on the device, every
// sweep of an iteration after `done` returns at once, and the host learns of
// convergence by polling a pinned copy of the status one check period behind
// the queue, so the GPU never waits for the host.
#include <cudaTypedefs.h>
#include <stdio.h>
#include <string.h>

#include <cmath>

#include "sk_internal.h"
#include "sk_solve.cuh"

namespace sk {

// ---------------------------------------------------------------------------
// Prologue of forward.py:119-156 on the device, one CTA per batch item:
// default marginals, log(clamp(., 1e-38)), f = g = 0 (or kept for a warm
// start), effective potentials (-inf at masked entries), valid index ranges,
// zeroed tickets and the status record.
struct InitArgs {
    int64_t B, N, M;
    const float* a;
    const float* b;
    const uint8_t* mask_a;
    const uint8_t* mask_b;
    float* log_a;
    float* log_b;
    float* f;
    float* g;
    float* f_eff;
    float* g_eff;
    int* ranges;
    unsigned* tickets;
    int64_t tickets_per_item;
    Status* st;
    int max_iters, check_every, decide;
    float threshold;
    int keep_potentials;
    int iter_masks;  // 0: masks only shape the default marginals
};

__device__ __forceinline__ void block_count_range(const uint8_t* mask, int64_t n,
                                                  float* cnt, int* lo, int* hi) {
    __shared__ float s_c[32];
    __shared__ int s_lo[32], s_hi[32];
    float c = 0.f;
    int l = INT32_MAX, h = -1;
    for (int64_t t = threadIdx.x; t < n; t += blockDim.x) {
        if (mask == nullptr || mask[t]) {
            c += 1.f;
            l = min(l, (int)t);
            h = max(h, (int)t);
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        c += __shfl_xor_sync(0xffffffffu, c, o);
        l = min(l, __shfl_xor_sync(0xffffffffu, l, o));
        h = max(h, __shfl_xor_sync(0xffffffffu, h, o));
    }
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        s_c[w] = c;
        s_lo[w] = l;
        s_hi[w] = h;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int q = 1; q < nw; ++q) {
            c += s_c[q];
            l = min(l, s_lo[q]);
            h = max(h, s_hi[q]);
        }
        s_c[0] = c;
        s_lo[0] = l;
        s_hi[0] = h;
    }
    __syncthreads();
    *cnt = s_c[0];
    *lo = s_lo[0];
    *hi = s_hi[0];
    __syncthreads();
}

__device__ __forceinline__ float clamp_log(float a) {
    // log(a.clamp(min=1e-38)); NaN stays NaN like torch.clamp
    return logf(a < kTiny ? kTiny : a);
}

__global__ void k_init(InitArgs a) {
    const int64_t b = blockIdx.x;
    float cnt_a, cnt_b;
    int lo_a, hi_a, lo_b, hi_b;
    block_count_range(a.mask_a ? a.mask_a + b * a.N : nullptr, a.N, &cnt_a, &lo_a, &hi_a);
    block_count_range(a.mask_b ? a.mask_b + b * a.M : nullptr, a.M, &cnt_b, &lo_b, &hi_b);
    // default marginals (forward.py:132-142): fp32 1/N, or mask / max(count, 1)
    const float inv_a = 1.f / (a.mask_a ? fmaxf(cnt_a, 1.f) : (float)a.N);
    const float inv_b = 1.f / (a.mask_b ? fmaxf(cnt_b, 1.f) : (float)a.M);
    for (int64_t t = threadIdx.x; t < a.N; t += blockDim.x) {
        const int64_t r = b * a.N + t;
        const bool valid = a.mask_a == nullptr || a.mask_a[r];
        const float av = a.a ? a.a[r] : (valid ? inv_a : 0.f);
        a.log_a[r] = clamp_log(av);
        const float fv = a.keep_potentials ? a.f[r] : 0.f;
        if (!a.keep_potentials) a.f[r] = 0.f;
        a.f_eff[r] = (valid || !a.iter_masks) ? fv : -INFINITY;
    }
    for (int64_t t = threadIdx.x; t < a.M; t += blockDim.x) {
        const int64_t c = b * a.M + t;
        const bool valid = a.mask_b == nullptr || a.mask_b[c];
        const float bv = a.b ? a.b[c] : (valid ? inv_b : 0.f);
        a.log_b[c] = clamp_log(bv);
        const float gv = a.keep_potentials ? a.g[c] : 0.f;
        if (!a.keep_potentials) a.g[c] = 0.f;
        a.g_eff[c] = (valid || !a.iter_masks) ? gv : -INFINITY;
    }
    for (int64_t t = threadIdx.x; t < a.tickets_per_item; t += blockDim.x)
        a.tickets[b * a.tickets_per_item + t] = 0u;
    if (b == 0) {
        // the column finish's group counters and residuals
        const int64_t ng = 2 * fin_groups(a.B * a.M);
        for (int64_t t = threadIdx.x; t < ng; t += blockDim.x) status_fin_count(a.st)[t] = 0u;
    }
    if (threadIdx.x == 0) {
        int* r = a.ranges + 4 * b;
        r[0] = !a.iter_masks ? 0 : (hi_a >= 0 ? lo_a : 0);
        r[1] = !a.iter_masks ? (int)a.N : (hi_a >= 0 ? hi_a + 1 : 0);
        r[2] = !a.iter_masks ? 0 : (hi_b >= 0 ? lo_b : 0);
        r[3] = !a.iter_masks ? (int)a.M : (hi_b >= 0 ? hi_b + 1 : 0);
        if (b == 0) {
            Status s{};
            s.iter = 0;
            s.done = a.max_iters <= 0 ? 1 : 0;
            s.n_iters = 0;
            s.converged = 0;
            s.res_bits = 0u;
            s.ticket = 0u;
            s.max_iters = a.max_iters;
            s.check_every = a.check_every;
            s.threshold = a.threshold;
            s.decide = a.decide;
            s.err = 0;
            *a.st = s;
            // the persistent solve's grid-barrier counter: its own cache line
            // in the status region (bytes 128-255)
            status_bar(a.st)[0] = 0u;
            *status_push_ticket(a.st) = 0u;
        }
    }
}

// ---------------------------------------------------------------------------
// Launch helpers

template <int VEC, typename T = float>
static void launch_row_vec(const SweepPlan& p, const RowArgs& ra, cudaStream_t s) {
    const int64_t rows = ra.B * ra.N;
    const int rpc = kRowThreads / p.tpr;
    const unsigned grid = (unsigned)((rows + rpc - 1) / rpc);
    switch (p.tpr) {
        case 32: launch_pdl(k_row_sweep<VEC, 32, T>, grid, dim3(kRowThreads), 0, s, ra); break;
        case 64: launch_pdl(k_row_sweep<VEC, 64, T>, grid, dim3(kRowThreads), 0, s, ra); break;
        case 128: launch_pdl(k_row_sweep<VEC, 128, T>, grid, dim3(kRowThreads), 0, s, ra); break;
        default: launch_pdl(k_row_sweep<VEC, 256, T>, grid, dim3(kRowThreads), 0, s, ra); break;
    }
}

void launch_row(const SweepPlan& p, const RowArgs& ra, cudaStream_t s) {
    if (p.bf16) launch_row_vec<4, uint16_t>(p, ra, s);  // bf16 plans are always 4-wide
    else if (p.vec == 4) launch_row_vec<4>(p, ra, s);
    else launch_row_vec<1>(p, ra, s);
}

// The tensor-fed column sweep needs more than the default 48 KB of dynamic
// shared memory; the attributes are set once per device.
static bool tma_col_ready() {
    static thread_local unsigned long long ready = 0;  // bit per device ordinal
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
    if (ready & (1ull << dev)) return true;
    if (cudaFuncSetAttribute(k_col_sweep_tma<kBulkStages>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kBulkSmem) != cudaSuccess ||
        cudaFuncSetAttribute(k_col_sweep_tma<kBulkStages>,
                             cudaFuncAttributePreferredSharedMemoryCarveout,
                             (int)cudaSharedmemCarveoutMaxShared) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    ready |= 1ull << dev;
    return true;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against the driver library).
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
        cudaGetLastError();
    }
    return fn;
}

// 3-D map (M, N, B) of C with 128 x 64 x 1 boxes; false if it cannot be encoded.
static bool col_tensor_map(const ColArgs& ca, CUtensorMap* map) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)ca.M, (cuuint64_t)ca.N, (cuuint64_t)ca.B};
    const int64_t sb = ca.B > 1 ? ca.sCb : ca.sCn * ca.N;
    const cuuint64_t strides[2] = {(cuuint64_t)(ca.sCn * 4), (cuuint64_t)(sb * 4)};
    const cuuint32_t box[3] = {128, (cuuint32_t)kBulkRows, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void*)ca.C, dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

void launch_col(const SweepPlan& p, const ColArgs& ca, cudaStream_t s) {
    const unsigned grid = (unsigned)(ca.B * p.nbands * p.ntiles);
    CUtensorMap map;
    if (p.bf16)
        launch_pdl(k_col_sweep<4, uint16_t>, grid, dim3(kColThreads), 0, s, ca);
    else if (p.col_tma && tma_col_ready() && col_tensor_map(ca, &map))
        launch_pdl(k_col_sweep_tma<kBulkStages>, grid, dim3(kBulkThreads), kBulkSmem, s, map, ca);
    else if (p.vec == 4) launch_pdl(k_col_sweep<4>, grid, dim3(kColThreads), 0, s, ca);
    else launch_pdl(k_col_sweep<1>, grid, dim3(kColThreads), 0, s, ca);
}

Scalars make_scalars(double eps, double tau_a, double tau_b) {
    // compute_rho (unbalanced.py:13-25): tau None / inf -> balanced
    auto rho = [&](double tau) { return std::isinf(tau) ? 0.0 : eps / (eps + tau); };
    Scalars s;
    s.k = (float)(1.0 / eps);
    s.eps = (float)eps;
    const double ra = rho(tau_a), rb = rho(tau_b);
    s.rho_a = (float)ra;
    s.omr_a = (float)(1.0 - ra);
    s.rho_b = (float)rb;
    s.omr_b = (float)(1.0 - rb);
    return s;
}

RowArgs make_row_args(const Problem& P, const SolveWs& w, const Scalars& sc,
                      const uint8_t* mask_a, float* f, const float* f_in) {
    RowArgs r{};
    r.C = P.C;
    r.sCb = P.sCb;
    r.sCn = P.sCn;
    r.sCm = P.sCm;
    r.B = P.B;
    r.N = P.N;
    r.M = P.M;
    r.g_eff = w.g_eff;
    r.f_in = f_in;
    r.f_out = f;
    r.f_eff = w.f_eff;
    r.log_a = w.log_a;
    r.mask_a = mask_a;
    r.ranges = w.ranges;
    r.lse_out = nullptr;
    r.k = sc.k;
    r.eps = sc.eps;
    r.rho = sc.rho_a;
    r.omr = sc.omr_a;
    r.guard = 1;
    r.plain = 0;
    r.st = (Status*)w.status;
    return r;
}

ColArgs make_col_args(const Problem& P, const SweepPlan& p, const SolveWs& w,
                      const Scalars& sc, const uint8_t* mask_b, float* g,
                      const float* g_in) {
    ColArgs c{};
    c.C = P.C;
    c.sCb = P.sCb;
    c.sCn = P.sCn;
    c.sCm = P.sCm;
    c.B = P.B;
    c.N = P.N;
    c.M = P.M;
    c.f_eff = w.f_eff;
    c.g_in = g_in;
    c.g_out = g;
    c.g_eff = w.g_eff;
    c.log_b = w.log_b;
    c.mask_b = mask_b;
    c.ranges = w.ranges;
    c.partial = w.partial;
    c.tickets = w.tickets;
    c.lse_out = nullptr;
    c.ntiles = p.ntiles;
    c.nbands = p.nbands;
    c.band_rows = p.band_rows;
    c.k = sc.k;
    c.eps = sc.eps;
    c.rho = sc.rho_b;
    c.omr = sc.omr_b;
    c.guard = 1;
    c.plain = 0;
    c.st = (Status*)w.status;
    return c;
}

// Per-thread, per-device pinned slots for non-blocking convergence polling.
struct Poller {
    int* host = nullptr;       // 2 slots x 16 ints (Status prefix)
    cudaEvent_t ev[2] = {nullptr, nullptr};
    bool ok = false;
};
static thread_local Poller g_pollers[64];

static Poller* get_poller() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    Poller& p = g_pollers[dev];
    if (!p.ok) {
        if (cudaHostAlloc((void**)&p.host, 2 * 64, cudaHostAllocPortable) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        for (int q = 0; q < 2; ++q)
            if (cudaEventCreateWithFlags(&p.ev[q], cudaEventDisableTiming) != cudaSuccess) {
                cudaGetLastError();
                return nullptr;
            }
        p.ok = true;
    }
    return &p;
}

// Enqueue up to max_iters iterations. With a threshold, poll the device's
// decision one check period behind the queue and stop enqueueing once it is
// done (sweeps already queued return immediately).
int run_solve(const Problem& P, const SweepPlan& p, const RowArgs& ra, const ColArgs& ca,
              int max_iters, int check_every, bool checks, cudaStream_t s, bool allow_poll,
              const SolveWs* fused_ws, const Scalars* sc) {
    const bool fused = p.fused && fused_ws && sc;
    Poller* pl = (checks && allow_poll) ? get_poller() : nullptr;
    const Status* dst = ca.st;
    int pending = 0, slot = 0;
    for (int it = 0; it < max_iters; ++it) {
        if (fused) {
            if (int e = launch_fused(P, p, *fused_ws, *sc, ra.mask_a, ra.f_out, s)) return e;
            if (int e = launch_col_finish(fused_ws->fparts, (int)p.chunks, P.B * P.M + 4, P.B,
                                          P.M, ca.mask_b,
                                          fused_ws->log_b, ca.g_out, fused_ws->g_eff, *sc,
                                          fused_ws->status, s))
                return e;
        } else {
            launch_row(p, ra, s);
            launch_col(p, ca, s);
            SK_LAUNCHED("sinkhorn sweep launch");
        }
        if (pl && (it + 1) % check_every == 0 && it + 1 < max_iters) {
            SK_CUDA(cudaMemcpyAsync(pl->host + 16 * slot, dst, 64, cudaMemcpyDeviceToHost, s));
            SK_CUDA(cudaEventRecord(pl->ev[slot], s));
            ++pending;
            if (pending == 2) {
                const int older = slot ^ 1;
                SK_CUDA(cudaEventSynchronize(pl->ev[older]));
                --pending;
                if (((volatile int*)pl->host)[16 * older + 1]) break;  // done
            }
            slot ^= 1;
        }
    }
    return SK_OK;
}

int read_status(const void* st, Status* out, cudaStream_t s) {
    Poller* pl = get_poller();
    if (pl) {
        SK_CUDA(cudaMemcpyAsync(pl->host, st, 64, cudaMemcpyDeviceToHost, s));
        SK_CUDA(cudaStreamSynchronize(s));
        memcpy(out, pl->host, 64);
    } else {
        SK_CUDA(cudaMemcpyAsync(out, st, 64, cudaMemcpyDeviceToHost, s));
        SK_CUDA(cudaStreamSynchronize(s));
    }
    return SK_OK;
}

int init_solve(const Problem& P, const SolveWs& w, const float* a, const float* b,
               const uint8_t* mask_a, const uint8_t* mask_b, float* f, float* g,
               int max_iters, int check_every, float thr, int decide, int keep,
               cudaStream_t s, int iter_masks) {
    InitArgs ia{};
    ia.B = P.B;
    ia.N = P.N;
    ia.M = P.M;
    ia.a = a;
    ia.b = b;
    ia.mask_a = mask_a;
    ia.mask_b = mask_b;
    ia.log_a = w.log_a;
    ia.log_b = w.log_b;
    ia.f = f;
    ia.g = g;
    ia.f_eff = w.f_eff;
    ia.g_eff = w.g_eff;
    ia.ranges = w.ranges;
    ia.tickets = w.tickets;
    ia.tickets_per_item = max_col_tiles(P.M);
    ia.st = (Status*)w.status;
    ia.max_iters = max_iters;
    ia.check_every = check_every;
    ia.decide = decide;
    ia.threshold = thr;
    ia.keep_potentials = keep;
    ia.iter_masks = iter_masks;
    k_init<<<(unsigned)P.B, 256, 0, s>>>(ia);
    SK_LAUNCHED("k_init launch");
    return SK_OK;
}

}  // namespace sk

using namespace sk;

extern "C" {

size_t sk_forward_workspace_bytes(int64_t B, int64_t N, int64_t M) {
    if (B <= 0 || N <= 0 || M <= 0) return 0;
    return carve_solve(nullptr, B, N, M).bytes;
}

// The whole solve; keep = 1 starts from the potentials already in f and g.
static int forward_solve(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                         int64_t sCn, int64_t sCm, const float* a, const float* b,
                         const uint8_t* mask_a, const uint8_t* mask_b, double epsilon,
                         double tau_a, double tau_b, int max_iters, double threshold,
                         int check_every, float* f, float* g, void* workspace,
                         size_t workspace_bytes, int* n_iters, int* converged, void* stream,
                         int keep, int bf16 = 0) {
    clear_error();
    if (int e = check_problem(C, B, N, M, epsilon)) return e;
    if (!f || !g) return fail(SK_ERR_ARG, "f and g must be non-NULL");
    if (max_iters < 0) return fail(SK_ERR_ARG, "max_iters must be >= 0");
    if (check_every < 1) return fail(SK_ERR_ARG, "check_every must be >= 1");
    const SolveWs w = carve_solve(workspace, B, N, M);
    if (!workspace || workspace_bytes < w.bytes)
        return fail(SK_ERR_WORKSPACE, "workspace smaller than sk_forward_workspace_bytes");
    cudaStream_t s = (cudaStream_t)stream;
    const Problem P{C, B, N, M, sCb, sCn, sCm};
    const SweepPlan p = bf16 ? make_plan_bf16(C, B, N, M, sCb, sCn, sCm)
                             : make_plan(C, B, N, M, sCb, sCn, sCm);
    if (bf16 && p.vec != 4)
        return fail(SK_ERR_LAYOUT, "a bf16 C needs unit column stride, 16-byte aligned rows "
                                   "(row and batch strides multiples of 4) and M % 4 == 0");
    const Scalars sc = make_scalars(epsilon, tau_a, tau_b);
    // threshold <= 0 (or NaN) can never be met: skip the checks entirely
    const bool checks = threshold > 0.0;
    const float thr = (float)threshold;
    if (int e = init_solve(P, w, a, b, mask_a, mask_b, f, g, max_iters,
                           checks ? check_every : 0, thr, 1, keep, s))
        return e;
    bool onchip = false;
    if (!bf16) {
        if (int e = try_onchip_solve(P, w, sc, mask_a, mask_b, f, g, max_iters,
                                     checks ? check_every : 0, thr, s, &onchip))
            return e;
    }
    // The loop of single-read steps (k_fused_iter + k_col_finish, chained by
    // programmatic dependent launch) rather than the one-launch persistent
    // solve: measured on B200 the loop is as fast or faster on every fused
    // shape (0.185 vs 0.219 ms per iteration at N = M = 16384); the
    // persistent solve stays available as sk_solver_solve.
    if (!onchip) {
        const RowArgs ra = make_row_args(P, w, sc, mask_a, f, f);
        const ColArgs ca = make_col_args(P, p, w, sc, mask_b, g, g);
        if (int e = run_solve(P, p, ra, ca, max_iters, check_every, checks, s, true, &w, &sc))
            return e;
    }
    Status hs;
    if (int e = read_status(w.status, &hs, s)) return e;
    if (n_iters) *n_iters = max_iters <= 0 ? 0 : (hs.done ? hs.n_iters : max_iters);
    if (converged) *converged = hs.converged;
    if (hs.err == 2)
        return fail(SK_ERR_TIMEOUT, "a sweep kernel gave up waiting for its copies");
    if (hs.err) return fail(SK_ERR_DEVICE, "a sweep kernel reported an error");
    return SK_OK;
}

int sk_forward(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb, int64_t sCn,
               int64_t sCm, const float* a, const float* b, const uint8_t* mask_a,
               const uint8_t* mask_b, double epsilon, double tau_a, double tau_b,
               int max_iters, double threshold, int check_every, float* f, float* g,
               void* workspace, size_t workspace_bytes, int* n_iters, int* converged,
               void* stream) {
    return forward_solve(C, B, N, M, sCb, sCn, sCm, a, b, mask_a, mask_b, epsilon, tau_a,
                         tau_b, max_iters, threshold, check_every, f, g, workspace,
                         workspace_bytes, n_iters, converged, stream, 0);
}

int sk_forward_warm(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                    int64_t sCn, int64_t sCm, const float* a, const float* b,
                    const uint8_t* mask_a, const uint8_t* mask_b, double epsilon, double tau_a,
                    double tau_b, int max_iters, double threshold, int check_every, float* f,
                    float* g, void* workspace, size_t workspace_bytes, int* n_iters,
                    int* converged, void* stream) {
    return forward_solve(C, B, N, M, sCb, sCn, sCm, a, b, mask_a, mask_b, epsilon, tau_a,
                         tau_b, max_iters, threshold, check_every, f, g, workspace,
                         workspace_bytes, n_iters, converged, stream, 1);
}

int sk_forward_bf16(const uint16_t* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                    int64_t sCn, int64_t sCm, const float* a, const float* b,
                    const uint8_t* mask_a, const uint8_t* mask_b, double epsilon, double tau_a,
                    double tau_b, int max_iters, double threshold, int check_every, float* f,
                    float* g, void* workspace, size_t workspace_bytes, int* n_iters,
                    int* converged, void* stream) {
    // the kernels read C through its element type; the plan only looks at
    // the address and the strides
    return forward_solve(reinterpret_cast<const float*>(C), B, N, M, sCb, sCn, sCm, a, b,
                         mask_a, mask_b, epsilon, tau_a, tau_b, max_iters, threshold,
                         check_every, f, g, workspace, workspace_bytes, n_iters, converged,
                         stream, 0, 1);
}

int sk_solver_init(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                   int64_t sCn, int64_t sCm, const float* a, const float* b,
                   const uint8_t* mask_a, const uint8_t* mask_b, int max_iters,
                   double threshold, int check_every, int decide, float* f, float* g,
                   void* workspace, size_t workspace_bytes, void* stream) {
    clear_error();
    if (int e = check_problem(C, B, N, M, 1.0)) return e;
    if (!f || !g) return fail(SK_ERR_ARG, "f and g must be non-NULL");
    if (max_iters < 0 || check_every < 0)
        return fail(SK_ERR_ARG, "max_iters and check_every must be >= 0");
    const SolveWs w = carve_solve(workspace, B, N, M);
    if (!workspace || workspace_bytes < w.bytes)
        return fail(SK_ERR_WORKSPACE, "workspace smaller than sk_forward_workspace_bytes");
    const Problem P{C, B, N, M, sCb, sCn, sCm};
    const bool checks = threshold > 0.0 && check_every > 0;
    return init_solve(P, w, a, b, mask_a, mask_b, f, g, max_iters, checks ? check_every : 0,
                      (float)threshold, decide ? 1 : 0, 0, (cudaStream_t)stream);
}

int sk_solver_row_sweep(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                        int64_t sCn, int64_t sCm, const uint8_t* mask_a, double epsilon,
                        double tau_a, float* f, void* workspace, size_t workspace_bytes,
                        void* stream) {
    if (int e = check_problem(C, B, N, M, epsilon)) return e;
    if (!f) return fail(SK_ERR_ARG, "f must be non-NULL");
    const SolveWs w = carve_solve(workspace, B, N, M);
    if (!workspace || workspace_bytes < w.bytes)
        return fail(SK_ERR_WORKSPACE, "workspace smaller than sk_forward_workspace_bytes");
    const Problem P{C, B, N, M, sCb, sCn, sCm};
    const SweepPlan p = make_plan(C, B, N, M, sCb, sCn, sCm);
    const Scalars sc = make_scalars(epsilon, tau_a, INFINITY);
    launch_row(p, make_row_args(P, w, sc, mask_a, f, f), (cudaStream_t)stream);
    SK_LAUNCHED("k_row_sweep launch");
    return SK_OK;
}

int sk_solver_col_sweep(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                        int64_t sCn, int64_t sCm, const uint8_t* mask_b, double epsilon,
                        double tau_b, float* g, void* workspace, size_t workspace_bytes,
                        void* stream) {
    if (int e = check_problem(C, B, N, M, epsilon)) return e;
    if (!g) return fail(SK_ERR_ARG, "g must be non-NULL");
    const SolveWs w = carve_solve(workspace, B, N, M);
    if (!workspace || workspace_bytes < w.bytes)
        return fail(SK_ERR_WORKSPACE, "workspace smaller than sk_forward_workspace_bytes");
    const Problem P{C, B, N, M, sCb, sCn, sCm};
    const SweepPlan p = make_plan(C, B, N, M, sCb, sCn, sCm);
    const Scalars sc = make_scalars(epsilon, INFINITY, tau_b);
    launch_col(p, make_col_args(P, p, w, sc, mask_b, g, g), (cudaStream_t)stream);
    SK_LAUNCHED("k_col_sweep launch");
    return SK_OK;
}

int sk_solver_status(const void* workspace, int* iter, int* done, int* n_iters,
                     int* converged, float* residual, void* stream) {
    if (!workspace) return fail(SK_ERR_ARG, "workspace is NULL");
    Status hs;
    if (int e = read_status(workspace, &hs, (cudaStream_t)stream)) return e;
    if (iter) *iter = hs.iter;
    if (done) *done = hs.done;
    if (n_iters) *n_iters = hs.n_iters;
    if (converged) *converged = hs.converged;
    if (residual) memcpy(residual, &hs.res_bits, sizeof(float));
    return SK_OK;
}

int sk_lse_row(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb, int64_t sCn,
               int64_t sCm, const float* g, double epsilon, float* out, void* stream) {
    clear_error();
    if (int e = check_problem(C, B, N, M, epsilon)) return e;
    if (!g || !out) return fail(SK_ERR_ARG, "g and out must be non-NULL");
    const SweepPlan p = make_plan(C, B, N, M, sCb, sCn, sCm);
    const Scalars sc = make_scalars(epsilon, INFINITY, INFINITY);
    RowArgs r{};
    r.C = C;
    r.sCb = sCb;
    r.sCn = sCn;
    r.sCm = sCm;
    r.B = B;
    r.N = N;
    r.M = M;
    r.g_eff = g;
    r.f_out = out;
    r.k = sc.k;
    r.eps = sc.eps;
    r.plain = 1;
    launch_row(p, r, (cudaStream_t)stream);
    SK_LAUNCHED("k_row_sweep launch");
    return SK_OK;
}

size_t sk_lse_col_workspace_bytes(int64_t B, int64_t N, int64_t M) {
    if (B <= 0 || N <= 0 || M <= 0) return 0;
    int64_t br;
    const int64_t nb = col_bands(B, N, M, &br);
    return align_up(sizeof(unsigned) * B * max_col_tiles(M)) +
           align_up(sizeof(float) * B * nb * M);
}

int sk_lse_col(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb, int64_t sCn,
               int64_t sCm, const float* f, double epsilon, float* out, void* workspace,
               size_t workspace_bytes, void* stream) {
    clear_error();
    if (int e = check_problem(C, B, N, M, epsilon)) return e;
    if (!f || !out) return fail(SK_ERR_ARG, "f and out must be non-NULL");
    if (!workspace || workspace_bytes < sk_lse_col_workspace_bytes(B, N, M))
        return fail(SK_ERR_WORKSPACE, "workspace smaller than sk_lse_col_workspace_bytes");
    cudaStream_t s = (cudaStream_t)stream;
    const SweepPlan p = make_plan(C, B, N, M, sCb, sCn, sCm);
    const Scalars sc = make_scalars(epsilon, INFINITY, INFINITY);
    unsigned* tickets = (unsigned*)workspace;
    float* partial =
        (float*)((char*)workspace + align_up(sizeof(unsigned) * B * max_col_tiles(M)));
    SK_CUDA(cudaMemsetAsync(tickets, 0, sizeof(unsigned) * B * max_col_tiles(M), s));
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
    c.k = sc.k;
    c.eps = sc.eps;
    c.plain = 1;
    launch_col(p, c, s);
    SK_LAUNCHED("k_col_sweep launch");
    return SK_OK;
}

}  // extern "C"
