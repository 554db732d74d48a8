// sk_onchip.cu -- the whole forward solve in one launch for problems whose
// cost matrix fits in one SM's shared memory.
//
// At such sizes every iteration of the two-sweep solve is two kernel launches
// of a few microseconds each, so the launches, not the arithmetic, set the
// time. Here CTA b stages C[b] (any strides) into shared memory once, keeps
// f, g, their masked copies and the log-marginals beside it, and runs the
// iterations of src/sinkhorn/triton/forward.py:161-186 on chip: the f-update
// (forward.py:14-49), then the g-update with the new f (forward.py:52-82),
// with the epilogues, masks and residuals of the sweep kernels (sk_sweep.cuh).
// Both updates give each thread one line (a row, or a column) -- or one slice
// of a line when there are fewer lines than threads, the slices merged through
// shared memory -- so every thread runs its own online LSE with no cross-lane
// step. C is stored with an odd row pitch, which keeps both a row walk across
// threads (stride pitch) and a column walk (stride 1) free of bank conflicts.
// The convergence check is over the whole batch (forward.py:177-179): at a
// check every CTA adds its residual to one of three
// rotating slots, meets the others at a grid barrier and reads the same
// maximum, so all CTAs stop at the same iteration; a slot is cleared two
// checks before its next use, after a barrier that every reader of its last
// use has passed. The barrier needs all CTAs resident at once: with checks the
// kernel is launched cooperatively (the launch fails instead of deadlocking
// when they do not fit, and the caller runs the two-sweep loop instead). Every
// barrier wait is bounded; a timeout records error 2 in the status record.
#include <cmath>

#include "sk_internal.h"
#include "sk_solve.cuh"

namespace sk {

constexpr int kOcThreads = 512;
constexpr int kOcWarps = kOcThreads / 32;
constexpr size_t kOcMaxSmem = 200 * 1024;
constexpr uint32_t kOcBarrierPolls = 1u << 24;  // x ~64 ns sleeps: about a second

struct OnchipArgs {
    const float* C;
    int64_t sCb, sCn, sCm;
    int64_t B, N, M;
    const float* log_a;     // (B,N) from k_init
    const float* log_b;     // (B,M)
    const uint8_t* mask_a;  // (B,N) or nullptr
    const uint8_t* mask_b;  // (B,M) or nullptr
    float* f;               // (B,N) in: starting potentials, out: result
    float* g;               // (B,M)
    float k, eps, rho_a, omr_a, rho_b, omr_b;
    int max_iters, check_every;  // check_every 0: no checks
    float threshold;
    Status* st;
};

__host__ __device__ inline int64_t onchip_pitch(int64_t M) { return M | 1; }

__host__ __device__ inline size_t onchip_smem_bytes(int64_t N, int64_t M) {
    return sizeof(float) * ((size_t)N * onchip_pitch(M) + 3 * N + 3 * M + 2 * kOcThreads) +
           (size_t)N + M + 16;
}

// One thread's online LSE over its slice of a line: elements e = r, r + RS,
// ... < len of x(e) = (pot(e) - C(e)) * k.
template <bool ROW>
__device__ __forceinline__ void line_slice_lse(const float* Cs, int64_t pitch, const float* pot,
                                               int64_t line, int r, int RS, int64_t len,
                                               float k, float& m, float& s) {
    for (int64_t e0 = r; e0 < len; e0 += 4 * (int64_t)RS) {
        float x[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t e = e0 + (int64_t)u * RS;
            if (e < len) {
                const float c = ROW ? Cs[line * pitch + e] : Cs[e * pitch + line];
                x[u] = (pot[e] - c) * k;
            } else {
                x[u] = -INFINITY;
            }
        }
        lse_fold<4>(m, s, x);
    }
}

// Block-wide max of a non-negative residual that keeps NaN.
__device__ __forceinline__ float block_max_nan(float v, float* red) {
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float r = warp_max(v);
    if (__any_sync(0xffffffffu, isnan(v))) r = NAN;
    __syncthreads();
    if (lane == 0) red[w] = r;
    __syncthreads();
    float rr = red[0];
    for (int q = 1; q < kOcWarps; ++q) rr = (red[q] > rr || isnan(red[q])) ? red[q] : rr;
    return rr;
}

// Bounded barrier over the grid's CTAs (all resident: cooperative launch).
__device__ bool grid_barrier(Status* st, int* sh_ok) {
    __syncthreads();
    if (threadIdx.x == 0) {
        volatile unsigned* gen = &st->bar_gen;
        const unsigned g0 = *gen;
        __threadfence();
        bool ok = true;
        if (atomicAdd(&st->bar_count, 1u) == gridDim.x - 1) {
            st->bar_count = 0u;
            __threadfence();
            atomicAdd(&st->bar_gen, 1u);
        } else {
            uint32_t i = 0;
            for (; i < kOcBarrierPolls; ++i) {
                if (*gen != g0) break;
                __nanosleep(64);
            }
            ok = i < kOcBarrierPolls;
        }
        __threadfence();
        *sh_ok = ok ? 1 : 0;
    }
    __syncthreads();
    return *sh_ok != 0;
}

__global__ void __launch_bounds__(kOcThreads, 1) k_onchip_solve(OnchipArgs a) {
    extern __shared__ __align__(16) float sm[];
    const int64_t b = blockIdx.x;
    const int64_t N = a.N, M = a.M;
    const int64_t P = onchip_pitch(M);
    float* Cs = sm;          // N x P (odd pitch)
    float* fe = Cs + N * P;  // f, -inf at masked rows
    float* fv = fe + N;      // f
    float* la = fv + N;      // log a
    float* ge = la + N;      // g, -inf at masked columns
    float* gv = ge + M;      // g
    float* lb = gv + M;      // log b
    float* pm = lb + M;      // slice partials (fewer lines than threads)
    float* ps = pm + kOcThreads;
    uint8_t* va = reinterpret_cast<uint8_t*>(ps + kOcThreads);
    uint8_t* vb = va + N;
    __shared__ float red[kOcWarps];
    __shared__ int sh_ok, sh_stop;
    const int tid = threadIdx.x;
    Status* st = a.st;
    const float k = a.k;

    // ---- stage C, potentials, marginals ----------------------------------
    const float* Cb = a.C + b * a.sCb;
    for (int64_t e = tid; e < N * M; e += kOcThreads) {
        const int64_t i = e / M, j = e - i * M;
        Cs[i * P + j] = Cb[i * a.sCn + j * a.sCm];
    }
    for (int64_t i = tid; i < N; i += kOcThreads) {
        const int64_t r = b * N + i;
        const bool v = a.mask_a == nullptr || a.mask_a[r] != 0;
        va[i] = v;
        fv[i] = a.f[r];
        fe[i] = v ? fv[i] : -INFINITY;
        la[i] = a.log_a[r];
    }
    for (int64_t j = tid; j < M; j += kOcThreads) {
        const int64_t c = b * M + j;
        const bool v = a.mask_b == nullptr || a.mask_b[c] != 0;
        vb[j] = v;
        gv[j] = a.g[c];
        ge[j] = v ? gv[j] : -INFINITY;
        lb[j] = a.log_b[c];
    }
    __syncthreads();

    // slices per line: a line per thread when there are enough lines
    const int RSr = N >= kOcThreads ? 1 : (int)(kOcThreads / N);  // per row
    const int RSc = M >= kOcThreads ? 1 : (int)(kOcThreads / M);  // per column
    const int per_r = kOcThreads / RSr, per_c = kOcThreads / RSc;
    int n_done = a.max_iters;
    bool conv = false, failed = false;
    int chk = 0;
    for (int it = 0; it < a.max_iters; ++it) {
        const bool check = a.check_every > 0 && ((it + 1) % a.check_every) == 0;
        float res = 0.f;
        // ---- f-update: row i, slice r of its columns ----------------------
        for (int64_t i0 = 0; i0 < N; i0 += per_r) {
            const int64_t i = i0 + tid % per_r;
            const int r = tid / per_r;
            float m = -INFINITY, s = 0.f;
            if (i < N && r < RSr && va[i])
                line_slice_lse<true>(Cs, P, ge, i, r, RSr, M, k, m, s);
            if (RSr > 1) {
                __syncthreads();  // the partials of the previous pass are read
                pm[tid] = m;
                ps[tid] = s;
                __syncthreads();
                if (r == 0 && i < N)
                    for (int q = 1; q < RSr; ++q) lse_merge(m, s, pm[q * per_r + tid], ps[q * per_r + tid]);
            }
            if (r == 0 && i < N) {
                const float fin = fv[i];
                float fo = 0.f;  // masked_fill(~mask_a, 0) (forward.py:168-169)
                if (va[i]) {
                    const float full = softmin_from_pair(m, s, a.eps, true) + a.eps * la[i];
                    fo = (a.rho_a == 0.f) ? full : a.rho_a * fin + a.omr_a * full;
                }
                fv[i] = fo;
                fe[i] = va[i] ? fo : -INFINITY;
                const float d = fabsf(fo - fin);
                res = (d > res || isnan(d)) ? d : res;
            }
        }
        __syncthreads();
        // ---- g-update with the new f: column j, slice r of its rows -------
        for (int64_t j0 = 0; j0 < M; j0 += per_c) {
            const int64_t j = j0 + tid % per_c;
            const int r = tid / per_c;
            float m = -INFINITY, s = 0.f;
            if (j < M && r < RSc) line_slice_lse<false>(Cs, P, fe, j, r, RSc, N, k, m, s);
            if (RSc > 1) {
                __syncthreads();
                pm[tid] = m;
                ps[tid] = s;
                __syncthreads();
                if (r == 0 && j < M)
                    for (int q = 1; q < RSc; ++q) lse_merge(m, s, pm[q * per_c + tid], ps[q * per_c + tid]);
            }
            if (r == 0 && j < M) {
                const float gin = gv[j];
                float go = 0.f;  // masked_fill(~mask_b, 0) (forward.py:170-171)
                if (vb[j]) {
                    const float full = softmin_from_pair(m, s, a.eps, true) + a.eps * lb[j];
                    go = (a.rho_b == 0.f) ? full : a.rho_b * gin + a.omr_b * full;
                }
                gv[j] = go;
                ge[j] = vb[j] ? go : -INFINITY;
                const float d = fabsf(go - gin);
                res = (d > res || isnan(d)) ? d : res;
            }
        }
        __syncthreads();
        // ---- convergence check over the whole batch (every check_every) --
        if (check) {
            const float r = block_max_nan(res, red);
            if (gridDim.x == 1) {
                if (tid == 0) sh_stop = r < a.threshold;
            } else {
                const int slot = chk % 3;
                if (tid == 0) atomic_max_nonneg(&st->res_slot[slot], r);
                if (!grid_barrier(st, &sh_ok)) {
                    failed = true;
                    break;
                }
                if (tid == 0) {
                    const float gr = __uint_as_float(atomicOr(&st->res_slot[slot], 0u));
                    sh_stop = gr < a.threshold;
                    if (blockIdx.x == 0) st->res_slot[(chk + 2) % 3] = 0u;
                }
            }
            ++chk;
            __syncthreads();
            if (sh_stop) {
                conv = true;
                n_done = it + 1;
                break;
            }
        }
    }
    __syncthreads();
    for (int64_t i = tid; i < N; i += kOcThreads) a.f[b * N + i] = fv[i];
    for (int64_t j = tid; j < M; j += kOcThreads) a.g[b * M + j] = gv[j];
    if (tid == 0) {
        if (failed) atomicMax(&st->err, 2);
        if (b == 0) {
            st->n_iters = n_done;
            st->converged = conv ? 1 : 0;
            st->iter = n_done;
            st->done = 1;
        }
    }
}

// Whether the problem qualifies (fp32 C of any strides, one item's C and
// vectors within kOcMaxSmem) and, if so, the launch; *ran reports whether it
// ran (false: run the two-sweep loop).
int try_onchip_solve(const Problem& P, const SolveWs& w, const Scalars& sc,
                     const uint8_t* mask_a, const uint8_t* mask_b, float* f, float* g,
                     int max_iters, int check_every, float thr, cudaStream_t s, bool* ran) {
    *ran = false;
    if (max_iters <= 0) return SK_OK;
    const size_t smem = onchip_smem_bytes(P.N, P.M);
    if (smem > kOcMaxSmem) return SK_OK;
    int dev = 0;
    SK_CUDA(cudaGetDevice(&dev));
    static thread_local unsigned long long ready = 0;
    if (!(ready & (1ull << (dev & 63)))) {
        SK_CUDA(cudaFuncSetAttribute(k_onchip_solve, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kOcMaxSmem));
        ready |= 1ull << (dev & 63);
    }
    OnchipArgs a{};
    a.C = P.C;
    a.sCb = P.sCb;
    a.sCn = P.sCn;
    a.sCm = P.sCm;
    a.B = P.B;
    a.N = P.N;
    a.M = P.M;
    a.log_a = w.log_a;
    a.log_b = w.log_b;
    a.mask_a = mask_a;
    a.mask_b = mask_b;
    a.f = f;
    a.g = g;
    a.k = sc.k;
    a.eps = sc.eps;
    a.rho_a = sc.rho_a;
    a.omr_a = sc.omr_a;
    a.rho_b = sc.rho_b;
    a.omr_b = sc.omr_b;
    a.max_iters = max_iters;
    a.check_every = check_every;
    a.threshold = thr;
    a.st = (Status*)w.status;
    const dim3 grid((unsigned)P.B), block(kOcThreads);
    if (check_every > 0 && P.B > 1) {
        // the checks meet at grid barriers: every CTA must be resident
        void* args[] = {&a};
        const cudaError_t e = cudaLaunchCooperativeKernel((const void*)k_onchip_solve, grid,
                                                          block, args, smem, s);
        if (e == cudaErrorCooperativeLaunchTooLarge) {
            cudaGetLastError();  // too many items to be resident at once
            return SK_OK;
        }
        if (e != cudaSuccess) return cuda_fail(e, "k_onchip_solve cooperative launch");
    } else {
        k_onchip_solve<<<grid, block, smem, s>>>(a);
        SK_LAUNCHED("k_onchip_solve launch");
    }
    *ran = true;
    return SK_OK;
}

}  // namespace sk
