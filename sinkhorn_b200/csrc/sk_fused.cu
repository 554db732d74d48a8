// sk_fused.cu -- one Sinkhorn iteration with a single read of C.
//
// f_new_i depends only on row i of C (and the previous g), so a row can be
// consumed twice while it sits in shared memory: first for its row LSE (the
// f-update), then -- with the f_new just computed -- for the column LSEs of the
// g-update. A cluster of two CTAs (one per SM) owns a chunk of rows; CTA q
// owns columns [q M/2, (q+1) M/2). For each row:
//   * a producer warp streams the CTA's half-row (M/2 fp32) into a 4-stage
//     ring with one cp.async.bulk;
//   * 16 consumer warps form the half-row's (max, sum exp) with a max pass and
//     an exp-sum pass (two named barriers), send the pair to the peer CTA
//     through distributed shared memory (st.shared::cluster + a remote
//     mbarrier arrive) and, while the peer's pair is in flight, fold the
//     previous row into their per-column running (max, sum) states -- one
//     exp per element, the states live in registers;
//   * after the peer's pair arrives (bounded wait) every thread holds the row
//     LSE and the new f_i.
// At the end of its rows each CTA writes one partial column LSE per column;
// k_col_finish (sk_shard.cu) merges the chunks, applies the g-update, the
// residual and the convergence decision. Gauss-Seidel order is that of
// src/sinkhorn/triton/forward.py:161-184; only the summation order differs.
//
// Every wait is bounded; a timeout sets an abort flag that all consumer warps
// observe after their next named barrier, the producer lets its copies land,
// and both CTAs meet at the final cluster barrier, so no path can hang or
// leave a CTA's shared memory reachable after it exits.
#include <cmath>

#include "sk_internal.h"
#include "sk_solve.cuh"
#include "sk_tma.cuh"

namespace sk {

constexpr int kFzConsumers = 512;
constexpr int kFzWarps = kFzConsumers / 32;
constexpr int kFzThreads = kFzConsumers + 32;  // + producer warp
constexpr int kFzStages = 4;

struct FusedArgs {
    const float* C;
    int64_t sCb, sCn;
    int64_t B, N, M;
    const float* g_eff;     // (B,M) previous g, -inf at masked columns
    const float* f_in;      // (B,N)
    float* f_out;           // (B,N)
    float* f_eff;           // (B,N)
    const float* log_a;     // (B,N)
    const uint8_t* mask_a;  // (B,N) or nullptr
    float* parts;           // (chunks, B*M + 4) column LSE partials (16-byte rows)
    int64_t chunks;         // row chunks per batch item
    int64_t rows_per_chunk;
    float k, eps, rho, omr;
    Status* st;
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ uint32_t map_to_rank(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}

__device__ __forceinline__ void st_remote_f32x2(uint32_t addr, float x, float y) {
    asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(x), "f"(y)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_remote(uint32_t addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(addr)
                 : "memory");
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

// Named barriers over the consumer warps only (the producer never joins
// them): id 2 plain, id 1 reducing.
__device__ __forceinline__ void consumer_sync() {
    asm volatile("barrier.sync 2, %0;" ::"n"(kFzConsumers) : "memory");
}

// Same barrier with an OR-reduction: every consumer gets the same answer, so
// a loop exit decided on it is uniform (no thread is left at a barrier).
__device__ __forceinline__ bool consumer_sync_or(bool pred) {
    uint32_t out;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "barrier.red.or.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(out)
        : "r"((uint32_t)pred), "n"(kFzConsumers)
        : "memory");
    return out != 0;
}

__device__ __forceinline__ bool wait_full(uint64_t* bar, uint32_t parity, volatile int* ab) {
    for (uint32_t i = 0; i < kWaitPolls; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*ab) return false;
    }
    return false;
}

__device__ __forceinline__ bool wait_peer(uint64_t* bar, uint32_t parity, volatile int* ab) {
    for (uint32_t i = 0; i < kWaitPolls; ++i) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if (*ab) return false;
    }
    return false;
}

// G4 = float4 column groups per consumer thread within the CTA's half-row.
template <int G4>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kFzThreads, 1)
    k_fused_iter(FusedArgs a) {
    constexpr int NV = 4 * G4;  // columns per consumer thread
    extern __shared__ __align__(128) unsigned char smem[];
    const int64_t half = a.M >> 1;
    float* ring = reinterpret_cast<float*>(smem);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)kFzStages * half * 4);
    uint64_t* empty = full + kFzStages;
    uint64_t* peer_bar = empty + kFzStages;                 // [2], arrived on by the peer
    float2* peer_pair = reinterpret_cast<float2*>(peer_bar + 2);  // [2], written by the peer
    __shared__ float wmax[kFzWarps], wsum[kFzWarps];
    __shared__ volatile int sh_abort;

    Status* st = a.st;
    if (read_volatile(&st->done)) return;  // both CTAs of a cluster read the same flag
    const bool check = is_check_iter(st, read_volatile(&st->iter));
    const uint32_t rank = cluster_ctarank();
    const uint32_t peer = rank ^ 1u;
    const int64_t unit = blockIdx.x >> 1;
    const int64_t b = unit / a.chunks;
    const int64_t chunk = unit - b * a.chunks;
    const int64_t r0 = chunk * a.rows_per_chunk;
    const int64_t r1 = (r0 + a.rows_per_chunk) < a.N ? (r0 + a.rows_per_chunk) : a.N;
    const int64_t R = r1 > r0 ? r1 - r0 : 0;
    const int64_t col0 = (int64_t)rank * half;

    if (threadIdx.x == 0) {
        for (int q = 0; q < kFzStages; ++q) {
            mbar_init(&full[q], 1);
            mbar_init(&empty[q], kFzWarps);
        }
        mbar_init(&peer_bar[0], 1);
        mbar_init(&peer_bar[1], 1);
        sh_abort = 0;
        mbar_init_fence();
    }
    __syncthreads();
    __syncwarp();
    cluster_barrier();  // the peer's barriers exist before any remote arrive

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp == kFzWarps) {
        // ---- producer: one bulk copy of the half-row per stage ----------
        if (lane == 0 && R > 0) {
            const float* src = a.C + b * a.sCb + r0 * a.sCn + col0;
            const uint32_t bytes = (uint32_t)(half * 4);
            int64_t issued = 0;
            for (int64_t i = 0; i < R; ++i) {
                const int q = (int)(i % kFzStages);
                if (i >= kFzStages &&
                    !wait_full(&empty[q], (uint32_t)((i / kFzStages) - 1) & 1u, &sh_abort)) {
                    sh_abort = 1;
                    break;
                }
                mbar_expect_tx(&full[q], bytes);
                bulk_g2s(ring + (size_t)q * half, src + i * a.sCn, bytes, &full[q]);
                issued = i + 1;
            }
            const int64_t first = issued > kFzStages ? issued - kFzStages : 0;
            for (int64_t i = first; i < issued; ++i)
                if (!mbar_wait(&full[i % kFzStages], (uint32_t)(i / kFzStages) & 1u))
                    sh_abort = 1;
        }
    } else {
        // ---- consumers ----------------------------------------------------
        const int tid = threadIdx.x;
        const float k = a.k;
        float gk[NV], cm[NV], cs[NV];
        bool gv[G4];
#pragma unroll
        for (int u = 0; u < G4; ++u) {
            const int64_t c4 = (int64_t)(tid + kFzConsumers * u) * 4;  // column in the half
            gv[u] = c4 < half;
            float4 g4 = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
            if (gv[u]) g4 = ld_vec4(a.g_eff + b * a.M + col0 + c4);
            gk[4 * u + 0] = g4.x;
            gk[4 * u + 1] = g4.y;
            gk[4 * u + 2] = g4.z;
            gk[4 * u + 3] = g4.w;
        }
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            cm[v] = -3.0e38f;  // finite start: an empty column keeps cs = 0
            cs[v] = 0.f;
        }
        float f_prev = -INFINITY;  // effective f of the previous row
        float res = 0.f;
        bool failed = false;       // this thread's own wait gave up
        const uint32_t remote_pair0 = map_to_rank(&peer_pair[0], peer);
        const uint32_t remote_bar0 = map_to_rank(&peer_bar[0], peer);
        for (int64_t i = 0; i <= R; ++i) {
            const bool have = i < R;
            float x[NV];
            float tmax = -INFINITY;
            // this row's scalars, loaded now so their latency hides behind the
            // row pass (they are needed only after the peer exchange)
            const int64_t grow = b * a.N + r0 + i;
            float fin = 0.f, lav = 0.f;
            bool valid = true;
            if (have) {
                fin = __ldg(a.f_in + grow);
                lav = __ldg(a.log_a + grow);
                valid = (a.mask_a == nullptr) || (a.mask_a[grow] != 0);
            }
            if (have) {
                const int q = (int)(i % kFzStages);
                if (!wait_full(&full[q], (uint32_t)(i / kFzStages) & 1u, &sh_abort)) failed = true;
                const float* row = ring + (size_t)q * half;
#pragma unroll
                for (int u = 0; u < G4; ++u) {
                    float4 c = make_float4(INFINITY, INFINITY, INFINITY, INFINITY);
                    if (gv[u]) c = *reinterpret_cast<const float4*>(row + (tid + kFzConsumers * u) * 4);
                    x[4 * u + 0] = (gk[4 * u + 0] - c.x) * k;
                    x[4 * u + 1] = (gk[4 * u + 1] - c.y) * k;
                    x[4 * u + 2] = (gk[4 * u + 2] - c.z) * k;
                    x[4 * u + 3] = (gk[4 * u + 3] - c.w) * k;
                }
#pragma unroll
                for (int v = 0; v < NV; ++v) tmax = fmaxf(tmax, x[v]);
                tmax = warp_max(tmax);
                if (lane == 0) wmax[warp] = tmax;
            }
            // (1) warp maxima visible; every consumer agrees on aborting
            if (consumer_sync_or(failed || sh_abort)) {
                sh_abort = 1;
                break;
            }
            float hmax = -INFINITY, hsum = 0.f;
            if (have) {
#pragma unroll
                hmax = lane < kFzWarps ? wmax[lane] : -INFINITY;
                hmax = warp_max(hmax);  // all 32 lanes end with the maximum
                float ts = 0.f;
                if (hmax != -INFINITY) {
#pragma unroll
                    for (int v = 0; v < NV; ++v) ts += expd(x[v] - hmax);
                }
                ts = warp_sum(ts);
                if (lane == 0) wsum[warp] = ts;
            }
            consumer_sync();  // (2) warp sums visible
            if (have) {
#pragma unroll
                hsum = lane < kFzWarps ? wsum[lane] : 0.f;
                hsum = warp_sum(hsum);  // all 32 lanes end with the sum
                if (tid == 0) {
                    // this half-row's (max, sum) to the peer, then signal it
                    st_remote_f32x2(remote_pair0 + (uint32_t)(i & 1) * sizeof(float2), hmax, hsum);
                    mbar_arrive_remote(remote_bar0 + (uint32_t)(i & 1) * sizeof(uint64_t));
                }
            }
            // fold the previous row into the column states with its new f
            if (i >= 1) {
                const int q = (int)((i - 1) % kFzStages);
                const float* row = ring + (size_t)q * half;
                if (f_prev != -INFINITY) {
#pragma unroll
                    for (int u = 0; u < G4; ++u) {
                        if (!gv[u]) continue;
                        const float4 c = *reinterpret_cast<const float4*>(row + (tid + kFzConsumers * u) * 4);
                        const float tv[4] = {f_prev - c.x, f_prev - c.y, f_prev - c.z,
                                             f_prev - c.w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            // online LSE with one exp: d = y - m; a new max rescales
                            // (and becomes y itself: m + d would lose y when m is the
                            // -3e38 starting value)
                            const int v = 4 * u + e;
                            const float y = tv[e] * k;
                            const float d = y - cm[v];
                            const float ex = ex2(-fabsf(d) * kLog2e);
                            if (d > 0.f) {
                                cs[v] = fmaf(cs[v], ex, 1.f);
                                cm[v] = y;
                            } else {
                                cs[v] += ex;
                            }
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[q]);
            }
            if (have) {
                if (!wait_peer(&peer_bar[i & 1], (uint32_t)((i >> 1) & 1), &sh_abort)) {
                    failed = true;
                    f_prev = -INFINITY;
                    continue;  // the next reducing barrier ends the loop
                }
                const float2 pp = peer_pair[i & 1];
                float mm = hmax, ss = hsum;
                lse_merge(mm, ss, pp.x, pp.y);
                float fo = 0.f;  // masked_fill(~mask_a, 0)
                if (valid) {
                    const float sm = softmin_from_pair(mm, ss, a.eps, true);
                    const float fullv = sm + a.eps * lav;
                    fo = (a.rho == 0.f) ? fullv : a.rho * fin + a.omr * fullv;
                }
                f_prev = valid ? fo : -INFINITY;
                if (rank == 0 && tid == 0) {
                    a.f_out[grow] = fo;
                    a.f_eff[grow] = f_prev;
                    const float d = fabsf(fo - fin);
                    res = (d > res || isnan(d)) ? d : res;
                }
            }
        }
        // this chunk's column partials (natural-log LSE per column)
        const int64_t pstride = a.B * a.M + 4;  // keeps every chunk row 16-byte aligned
        float* dst = a.parts + chunk * pstride + b * a.M + col0;
#pragma unroll
        for (int u = 0; u < G4; ++u) {
            if (!gv[u]) continue;
            const int64_t c4 = (int64_t)(tid + kFzConsumers * u) * 4;
            float4 o;
            o.x = cs[4 * u + 0] > 0.f ? cm[4 * u + 0] + logf(cs[4 * u + 0]) : -INFINITY;
            o.y = cs[4 * u + 1] > 0.f ? cm[4 * u + 1] + logf(cs[4 * u + 1]) : -INFINITY;
            o.z = cs[4 * u + 2] > 0.f ? cm[4 * u + 2] + logf(cs[4 * u + 2]) : -INFINITY;
            o.w = cs[4 * u + 3] > 0.f ? cm[4 * u + 3] + logf(cs[4 * u + 3]) : -INFINITY;
            *reinterpret_cast<float4*>(dst + c4) = o;
        }
        if (tid == 0 && rank == 0) {
            if (b == 0) a.parts[chunk * pstride + a.B * a.M] = 0.f;
            if (check) atomic_max_nonneg(&st->res_bits, res);
            if (sh_abort || failed) atomicMax(&st->err, 2);
        }
    }
    __syncthreads();
    __syncwarp();
    cluster_barrier();  // no CTA leaves while its peer may still touch its shared memory
}

// Opt in to more than 48 KB of dynamic shared memory, once per device.
template <int G4>
static int ensure_fused_smem() {
    static thread_local unsigned long long ready = 0;  // bit per device ordinal
    int dev = 0;
    SK_CUDA(cudaGetDevice(&dev));
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(ready & bit)) {
        SK_CUDA(cudaFuncSetAttribute(k_fused_iter<G4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)(kFzStages * 8192 * 4 + 256)));
        SK_CUDA(cudaFuncSetAttribute(k_fused_iter<G4>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     (int)cudaSharedmemCarveoutMaxShared));
        ready |= bit;
    }
    return SK_OK;
}

template <int G4>
static int launch_fused_g(const FusedArgs& a, int64_t nunits, cudaStream_t s) {
    const size_t smem = (size_t)kFzStages * (a.M / 2) * 4 + 2 * kFzStages * 8 + 2 * 8 + 2 * 8;
    if (int e = ensure_fused_smem<G4>()) return e;
    k_fused_iter<G4><<<(unsigned)(2 * nunits), kFzThreads, smem, s>>>(a);
    SK_LAUNCHED("k_fused_iter launch");
    return SK_OK;
}

}  // namespace sk

namespace sk {

// Co-resident 2-CTA clusters of k_fused_iter on the current device (cached);
// B200 gives ~74 (one CTA per SM, all SMs paired within their GPCs).
static int fused_active_clusters() {
    static thread_local int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 74;
    if (cache[dev] > 0) return cache[dev];
    int n = 0;
    const int smem = kFzStages * 8192 * 4 + 256;
    if (ensure_fused_smem<4>() == SK_OK) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * 148, 1, 1);
        cfg.blockDim = dim3(kFzThreads, 1, 1);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, k_fused_iter<4>, &cfg) != cudaSuccess) n = 0;
    }
    cudaGetLastError();
    if (n <= 0) n = 74;
    cache[dev] = n;
    return n;
}

int64_t fused_max_chunks(int64_t B) {
    return B >= 296 ? 1 : (296 + B - 1) / B;
}

void plan_fused(SweepPlan& p, int64_t B, int64_t N, int64_t M) {
    p.fused = 0;
    p.fused_ok = 0;
    if (M % 8 != 0 || M < 2048 || M > 16384 || N < 1) return;
    const int64_t A = fused_active_clusters();
    const int64_t cmax = fused_max_chunks(B);
    int64_t best_c = 1;
    double best_eff = -1.0;
    for (int64_t c = 1; c <= cmax; ++c) {
        if (c > 1 && N / c < 16) break;  // keep chunks at least 16 rows deep
        const int64_t units = B * c;
        const int64_t waves = (units + A - 1) / A;
        const double eff = (double)units / (double)(A * waves);
        if (eff > best_eff + 1e-9) {
            best_eff = eff;
            best_c = c;
        }
    }
    p.rows_per_chunk = (N + best_c - 1) / best_c;
    p.chunks = (N + p.rows_per_chunk - 1) / p.rows_per_chunk;
    p.fused_ok = 1;
    // Measured on B200 at N=M=16384: 0.57-0.62 ms per fused iteration against
    // 0.41 ms for the two sweeps (the per-row exchange chain leaves the SM
    // idle), so sk_forward keeps the two-sweep kernels; the fused iteration
    // stays available through sk_solver_fused_step / _finish.
    p.fused = 0;
}

int launch_fused(const Problem& P, const SweepPlan& p, const SolveWs& w, const Scalars& sc,
                 const uint8_t* mask_a, float* f, cudaStream_t s) {
    FusedArgs a{};
    a.C = P.C;
    a.sCb = P.sCb;
    a.sCn = P.sCn;
    a.B = P.B;
    a.N = P.N;
    a.M = P.M;
    a.g_eff = w.g_eff;
    a.f_in = f;
    a.f_out = f;
    a.f_eff = w.f_eff;
    a.log_a = w.log_a;
    a.mask_a = mask_a;
    a.parts = w.fparts;
    a.chunks = p.chunks;
    a.rows_per_chunk = p.rows_per_chunk;
    a.k = sc.k;
    a.eps = sc.eps;
    a.rho = sc.rho_a;
    a.omr = sc.omr_a;
    a.st = (Status*)w.status;
    const int64_t nunits = P.B * p.chunks;
    const int64_t g4 = (P.M / 8 + kFzConsumers - 1) / kFzConsumers;
    if (g4 <= 1) return launch_fused_g<1>(a, nunits, s);
    if (g4 <= 2) return launch_fused_g<2>(a, nunits, s);
    return launch_fused_g<4>(a, nunits, s);  // M <= 16384: at most 4 groups per thread
}

}  // namespace sk

using namespace sk;

extern "C" {

int sk_plan_query(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb, int64_t sCn,
                  int64_t sCm, int* vec, int* fused, int64_t* chunks) {
    if (int e = check_problem(C, B, N, M, 1.0)) return e;
    const SweepPlan p = make_plan(C, B, N, M, sCb, sCn, sCm);
    if (vec) *vec = p.vec;
    if (fused) *fused = p.fused ? 2 : (p.fused_ok ? 1 : 0);
    if (chunks) *chunks = p.chunks;
    return SK_OK;
}

int sk_solver_fused_step(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
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
    if (!p.fused_ok) return fail(SK_ERR_LAYOUT, "this shape / layout has no fused iteration");
    const Scalars sc = make_scalars(epsilon, tau_a, INFINITY);
    return launch_fused(P, p, w, sc, mask_a, f, (cudaStream_t)stream);
}

int sk_solver_fused_finish(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                           int64_t sCn, int64_t sCm, const uint8_t* mask_b, double epsilon,
                           double tau_b, float* g, void* workspace, size_t workspace_bytes,
                           void* stream) {
    if (int e = check_problem(C, B, N, M, epsilon)) return e;
    if (!g) return fail(SK_ERR_ARG, "g must be non-NULL");
    const SolveWs w = carve_solve(workspace, B, N, M);
    if (!workspace || workspace_bytes < w.bytes)
        return fail(SK_ERR_WORKSPACE, "workspace smaller than sk_forward_workspace_bytes");
    const SweepPlan p = make_plan(C, B, N, M, sCb, sCn, sCm);
    if (!p.fused_ok) return fail(SK_ERR_LAYOUT, "this shape / layout has no fused iteration");
    const Scalars sc = make_scalars(epsilon, INFINITY, tau_b);
    return launch_col_finish(w.fparts, (int)p.chunks, B * M + 4, B, M, mask_b, w.log_b, g,
                             w.g_eff, sc, w.status, (cudaStream_t)stream);
}

}  // extern "C"
