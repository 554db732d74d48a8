// sk_shard.cu -- the column half-step of a row-sharded solve.
//
// When C is split by rows over P ranks, rank r holds rows [r0, r1) with its
// slice of f and a full copy of g. The f-update needs nothing from the other
// ranks; the column LSE of the g-update is a merge of the P per-rank column
// LSEs. So one iteration is
//   sk_solver_row_sweep      (local rows, as on one GPU)
//   sk_solver_col_partial    (the column LSE over the local rows: B*M floats,
//                             plus the local |delta f| residual in slot B*M)
//   all-gather of the P partial vectors (the caller's collective, e.g. NCCL)
//   sk_solver_col_finish     (merge, softmin, rho-mix, mask, residual, check)
// Every rank runs the finish on identical gathered data, so every rank takes
// the same convergence decision without another collective.
#include <algorithm>
#include <cmath>

#include "sk_grid.cuh"
#include "sk_internal.h"
#include "sk_merge.cuh"
#include "sk_solve.cuh"

namespace sk {

struct FinishArgs {
    const float* parts;  // (P, stride): P column-LSE vectors, residual at [B*M]
    int P;
    // pair input instead of partials (the all-reduce merge of a row-sharded
    // solve): column j's LSE is pair_m[j] + log(pair_s[j]); pair_m[B*M] holds
    // the ranks' largest f residual
    const float* pair_m;
    const float* pair_s;
    int64_t stride;
    int64_t B, M;
    const uint8_t* mask_b;
    const float* log_b;
    float* g;
    float* g_eff;
    float eps, rho, omr;
    Status* st;
    // peer input (the row-sharded exchange of sk_peer.cu): before merging,
    // wait (bounded) until every rank's flag holds this iteration + 1; the
    // vectors of iteration `iter` sit at parts + (iter & 1) * par_stride
    const unsigned* wait_flags;
    int64_t par_stride;
    const float* g_in;   // the previous g (nullptr: g itself)
    float* lse_out;      // (B,M) the merged column LSEs (natural log), or nullptr
    int guard;           // 1: an infinite softmin becomes 0 (the forward's guard)
};

constexpr int kFinCols = (int)kFinColsPerCta;  // columns per CTA: two groups of 32 lanes
constexpr int kFinishThreads = 2 * kMergeSubsets * 32;

// One CTA finishes 64 consecutive columns. Warp w takes column group w / 4
// and merge subset w % 4 of every column of its group (sk_merge.cuh: all of
// the subset's loads in flight, folded in a fixed order); the subset-0 warp
// of each group then merges the four subset pairs in order and applies the
// g-update, so the result does not depend on timing and equals the merge
// phase of the persistent solve bit for bit.
//
// What the previous iteration left (the status record, g) and the constants
// (mask_b, log b) are read before pdl_wait(): the only writer of the status
// and of g is the previous launch of this kernel, which completed before the
// kernel producing the partials passed its own pdl_wait() and let this launch
// start. Only the partials are waited for.
__global__ void __launch_bounds__(kFinishThreads) k_col_finish(FinishArgs a) {
    pdl_trigger();
    __shared__ float2 sh_pair[2][kMergeSubsets][32];
    __shared__ int sh_arrived;
    Status* st = a.st;
    if (read_volatile(&st->done)) return;
    const int iter = read_volatile(&st->iter);
    const bool check = is_check_iter(st, iter);
    const int64_t BM = a.B * a.M;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int cg = w / kMergeSubsets, sub = w % kMergeSubsets;
    const int64_t col = (int64_t)blockIdx.x * kFinCols + cg * 32 + lane;
    const unsigned grp = blockIdx.x / kFinGroupCtas;
    unsigned* gcount = status_fin_count(st);
    unsigned* gres = status_fin_res(st, BM);
    float gin = 0.f, lb = 0.f;
    bool valid = false;
    if (sub == 0 && col < BM) {
        gin = a.g_in ? a.g_in[col] : a.g[col];
        valid = (a.mask_b == nullptr) || (a.mask_b[col] != 0);
        lb = valid ? a.log_b[col] : 0.f;
    }
    pdl_wait();
    const float* parts = a.parts;
    bool arrived = true;
    if (a.wait_flags != nullptr) {
        if (threadIdx.x == 0) {
            sh_arrived = peer_wait_flags(a.wait_flags, a.P, (unsigned)iter + 1u) ? 1 : 0;
            if (!sh_arrived) atomicMax(&st->err, 2);  // a rank never delivered
        }
        __syncthreads();
        arrived = sh_arrived != 0;
        parts += (int64_t)(iter & 1) * a.par_stride;
    }
    if (a.pair_m == nullptr)
        sh_pair[cg][sub][lane] =
            merge_subset<false>(parts + col, a.stride, a.P, sub, col < BM && arrived);
    else if (sub == 0)
        sh_pair[cg][0][lane] = col < BM ? make_float2(a.pair_m[col], a.pair_s[col])
                                        : make_float2(-INFINITY, 0.f);
    __syncthreads();
    if (sub == 0 && arrived) {
        float res = 0.f;
        if (col < BM) {
            float mm, ss;
            if (a.pair_m == nullptr) {
                const float2 sp[kMergeSubsets] = {sh_pair[cg][0][lane], sh_pair[cg][1][lane],
                                                  sh_pair[cg][2][lane], sh_pair[cg][3][lane]};
                merge_subsets(mm, ss, sp);
            } else {
                mm = sh_pair[cg][0][lane].x;
                ss = sh_pair[cg][0][lane].y;
            }
            float go = 0.f;  // masked_fill(~mask_b, 0)
            if (valid) {
                const float sm = softmin_from_pair(mm, ss, a.eps, a.guard != 0);
                const float full = sm + a.eps * lb;
                go = (a.rho == 0.f) ? full : a.rho * gin + a.omr * full;
            }
            a.g[col] = go;
            a.g_eff[col] = valid ? go : -INFINITY;
            if (a.lse_out) a.lse_out[col] = lse_of(mm, ss);
            res = fabsf(go - gin);
        }
        if (check) {
            if (blockIdx.x == 0 && cg == 0) {
                // the parts' f residuals (or the ranks' largest, in pair input)
                if (a.pair_m != nullptr) {
                    const float rf = lane == 0 ? a.pair_m[BM] : 0.f;
                    res = (rf > res || isnan(rf)) ? rf : res;
                } else {
                    for (int p = lane; p < a.P; p += 32) {
                        const float rf = parts[(int64_t)p * a.stride + BM];
                        res = (rf > res || isnan(rf)) ? rf : res;
                    }
                }
            }
            float r = warp_max(res);
            if (__any_sync(0xffffffffu, isnan(res))) r = NAN;
            if (lane == 0) atomic_max_nonneg(&gres[grp], r);
        }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        // arrive in this CTA's group; the group's last CTA carries the group's
        // residual to the Status record and arrives at the Status ticket
        const unsigned gsize = min((unsigned)kFinGroupCtas, gridDim.x - grp * kFinGroupCtas);
        const unsigned ngroups = (gridDim.x + kFinGroupCtas - 1) / kFinGroupCtas;
        if (atomicAdd(&gcount[grp], 1u) == gsize - 1) {
            gcount[grp] = 0u;
            __threadfence();
            if (check) atomic_max_nonneg(&st->res_bits, __uint_as_float(atomicExch(&gres[grp], 0u)));
            __threadfence();
            const unsigned prev = atomicAdd(&st->ticket, 1u);
            if (prev == ngroups - 1) {
                __threadfence();
                st->ticket = 0u;
                if (check) {
                    const float r = __uint_as_float(atomicOr(&st->res_bits, 0u));
                    if (st->decide && r < st->threshold) {
                        st->converged = 1;
                        st->done = 1;
                        st->n_iters = iter + 1;
                    }
                    if (st->decide) st->res_bits = 0u;
                }
                const int next = iter + 1;
                st->iter = next;
                if (!st->done && next >= st->max_iters) {
                    st->done = 1;
                    st->n_iters = next;
                }
                __threadfence();
            }
        }
    }
}

// A rank's column LSE over its own rows (the row-sharded solve on the
// single-read step): the chunk partials of sk_solver_fused_step merged in the
// fixed order of sk_merge.cuh, out[j] = LSE (natural log, -inf for no term),
// and out[B*M] = this rank's f residual of a check iteration (0 otherwise; a
// NaN written as +inf, which never passes the threshold either and survives
// a float MAX reduction).
struct ChunkMergeArgs {
    const float* parts;
    int P;
    int64_t stride, BM;
    float* out;
    const Status* st;
};

__global__ void __launch_bounds__(kFinishThreads) k_chunk_merge(ChunkMergeArgs a) {
    pdl_trigger();
    __shared__ float2 sh_pair[2][kMergeSubsets][32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int cg = w / kMergeSubsets, sub = w % kMergeSubsets;
    const int64_t col = (int64_t)blockIdx.x * kFinCols + cg * 32 + lane;
    pdl_wait();
    sh_pair[cg][sub][lane] = merge_subset<false>(a.parts + col, a.stride, a.P, sub, col < a.BM);
    __syncthreads();
    if (sub == 0 && col < a.BM) {
        const float2 sp[kMergeSubsets] = {sh_pair[cg][0][lane], sh_pair[cg][1][lane],
                                          sh_pair[cg][2][lane], sh_pair[cg][3][lane]};
        float mm, ss;
        merge_subsets(mm, ss, sp);
        a.out[col] = lse_of(mm, ss);
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        const int iter = read_volatile(&a.st->iter);
        float r = 0.f;
        if (is_check_iter(a.st, iter)) r = __uint_as_float(read_volatile((const int*)&a.st->res_bits));
        a.out[a.BM] = isnan(r) ? INFINITY : r;
    }
}

// out[j] = exp(local[j] - gmax[j]) (0 where the global max is -inf): a rank's
// share of the column sums against the ranks' common max.
__global__ void k_rank_rescale(const float* local, const float* gmax, float* out, int64_t n) {
    pdl_trigger();
    pdl_wait();
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n;
         j += (int64_t)gridDim.x * blockDim.x) {
        const float m = gmax[j];
        out[j] = m == -INFINITY ? 0.f : expd(local[j] - m);
    }
}

// The convergence decision of a solve whose residual was reduced across
// ranks (decide = 0 kernels, then an all-reduce of res_bits): converged when
// the reduced residual of the check iteration just run is below the
// threshold (NaN never is); res_bits is cleared for the next check.
__global__ void k_decide(Status* st) {
    pdl_wait();
    if (threadIdx.x != 0 || st->done) return;
    const int iter = st->iter;  // iterations run so far
    if (iter > 0 && is_check_iter(st, iter - 1)) {
        const float r = __uint_as_float(st->res_bits);
        if (r < st->threshold) {
            st->converged = 1;
            st->done = 1;
            st->n_iters = iter;
        }
        st->res_bits = 0u;
    }
}

int launch_col_finish(const float* parts, int nparts, int64_t stride, int64_t B, int64_t M,
                      const uint8_t* mask_b, const float* log_b, float* g, float* g_eff,
                      const Scalars& sc, void* status, cudaStream_t s, const float* g_in,
                      float* lse_out, int guard) {
    FinishArgs a{};
    a.g_in = g_in;
    a.lse_out = lse_out;
    a.guard = guard;
    a.parts = parts;
    a.P = nparts;
    a.stride = stride;
    a.B = B;
    a.M = M;
    a.mask_b = mask_b;
    a.log_b = log_b;
    a.g = g;
    a.g_eff = g_eff;
    a.eps = sc.eps;
    a.rho = sc.rho_b;
    a.omr = sc.omr_b;
    a.st = (Status*)status;
    const int64_t grid = (B * M + kFinCols - 1) / kFinCols;
    launch_pdl(k_col_finish, dim3((unsigned)grid), dim3(kFinishThreads), 0, s, a);
    SK_LAUNCHED("k_col_finish launch");
    return SK_OK;
}

int launch_col_finish_peer(const float* parts, int nparts, int64_t stride, int64_t par_stride,
                           const unsigned* flags, int64_t B, int64_t M, const uint8_t* mask_b,
                           const float* log_b, float* g, float* g_eff, const Scalars& sc,
                           void* status, cudaStream_t s) {
    FinishArgs a{};
    a.parts = parts;
    a.P = nparts;
    a.stride = stride;
    a.B = B;
    a.M = M;
    a.mask_b = mask_b;
    a.log_b = log_b;
    a.g = g;
    a.g_eff = g_eff;
    a.eps = sc.eps;
    a.rho = sc.rho_b;
    a.omr = sc.omr_b;
    a.st = (Status*)status;
    a.wait_flags = flags;
    a.par_stride = par_stride;
    a.guard = 1;
    const int64_t grid = (B * M + kFinCols - 1) / kFinCols;
    launch_pdl(k_col_finish, dim3((unsigned)grid), dim3(kFinishThreads), 0, s, a);
    SK_LAUNCHED("k_col_finish launch");
    return SK_OK;
}

int launch_col_finish_pairs(const float* pair_m, const float* pair_s, int64_t B, int64_t M,
                            const uint8_t* mask_b, const float* log_b, float* g, float* g_eff,
                            const Scalars& sc, void* status, cudaStream_t s) {
    FinishArgs a{};
    a.guard = 1;
    a.pair_m = pair_m;
    a.pair_s = pair_s;
    a.P = 1;
    a.stride = B * M + 1;
    a.B = B;
    a.M = M;
    a.mask_b = mask_b;
    a.log_b = log_b;
    a.g = g;
    a.g_eff = g_eff;
    a.eps = sc.eps;
    a.rho = sc.rho_b;
    a.omr = sc.omr_b;
    a.st = (Status*)status;
    const int64_t grid = (B * M + kFinCols - 1) / kFinCols;
    launch_pdl(k_col_finish, dim3((unsigned)grid), dim3(kFinishThreads), 0, s, a);
    SK_LAUNCHED("k_col_finish launch");
    return SK_OK;
}

}  // namespace sk

using namespace sk;

extern "C" {

int sk_solver_col_partial(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                          int64_t sCn, int64_t sCm, double epsilon, float* partial,
                          void* workspace, size_t workspace_bytes, void* stream) {
    if (int e = check_problem(C, B, N, M, epsilon)) return e;
    if (!partial) return fail(SK_ERR_ARG, "partial must be non-NULL");
    const SolveWs w = carve_solve(workspace, B, N, M);
    if (!workspace || workspace_bytes < w.bytes)
        return fail(SK_ERR_WORKSPACE, "workspace smaller than sk_forward_workspace_bytes");
    const Problem P{C, B, N, M, sCb, sCn, sCm};
    const SweepPlan p = make_plan(C, B, N, M, sCb, sCn, sCm);
    const Scalars sc = make_scalars(epsilon, INFINITY, INFINITY);
    ColArgs c = make_col_args(P, p, w, sc, nullptr, partial, nullptr);
    c.g_eff = nullptr;
    c.plain = 2;
    launch_col(p, c, (cudaStream_t)stream);
    SK_LAUNCHED("k_col_sweep launch (partial)");
    return SK_OK;
}

int sk_solver_col_finish(const float* parts, int P, int64_t B, int64_t N, int64_t M,
                         const uint8_t* mask_b, double epsilon, double tau_b, float* g,
                         void* workspace, size_t workspace_bytes, void* stream) {
    if (!parts || !g) return fail(SK_ERR_ARG, "parts and g must be non-NULL");
    if (P < 1 || P > 256 || B <= 0 || N <= 0 || M <= 0)
        return fail(SK_ERR_ARG, "bad P (1..256), B, N or M");
    if (!(epsilon > 0.0)) return fail(SK_ERR_ARG, "epsilon must be positive");
    const SolveWs w = carve_solve(workspace, B, N, M);
    if (!workspace || workspace_bytes < w.bytes)
        return fail(SK_ERR_WORKSPACE, "workspace smaller than sk_forward_workspace_bytes");
    const Scalars sc = make_scalars(epsilon, INFINITY, tau_b);
    return launch_col_finish(parts, P, B * M + 1, B, M, mask_b, w.log_b, g, w.g_eff, sc,
                             w.status, (cudaStream_t)stream);
}

int sk_solver_chunk_merge(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                          int64_t sCn, int64_t sCm, float* out, void* workspace,
                          size_t workspace_bytes, void* stream) {
    if (int e = check_problem(C, B, N, M, 1.0)) return e;
    if (!out) return fail(SK_ERR_ARG, "out must be non-NULL");
    const SolveWs w = carve_solve(workspace, B, N, M);
    if (!workspace || workspace_bytes < w.bytes)
        return fail(SK_ERR_WORKSPACE, "workspace smaller than sk_forward_workspace_bytes");
    const SweepPlan p = make_plan(C, B, N, M, sCb, sCn, sCm);
    if (!p.fused_ok) return fail(SK_ERR_LAYOUT, "this shape / layout has no fused iteration");
    ChunkMergeArgs a{};
    a.parts = w.fparts;
    a.P = (int)p.chunks;
    a.stride = B * M + 4;
    a.BM = B * M;
    a.out = out;
    a.st = (const Status*)w.status;
    launch_pdl(k_chunk_merge, dim3((unsigned)((B * M + kFinCols - 1) / kFinCols)),
               dim3(kFinishThreads), 0, (cudaStream_t)stream, a);
    SK_LAUNCHED("k_chunk_merge launch");
    return SK_OK;
}

int sk_solver_rank_rescale(const float* local, const float* gmax, float* out, int64_t n,
                           void* stream) {
    if (!local || !gmax || !out) return fail(SK_ERR_ARG, "NULL argument");
    if (n <= 0) return fail(SK_ERR_ARG, "n must be positive");
    const int64_t blocks = std::min<int64_t>((n + 255) / 256, 148 * 8);
    launch_pdl(k_rank_rescale, dim3((unsigned)blocks), dim3(256), 0, (cudaStream_t)stream, local,
               gmax, out, n);
    SK_LAUNCHED("k_rank_rescale launch");
    return SK_OK;
}

int sk_solver_col_finish_pairs(const float* pair_m, const float* pair_s, int64_t B, int64_t N,
                               int64_t M, const uint8_t* mask_b, double epsilon, double tau_b,
                               float* g, void* workspace, size_t workspace_bytes,
                               void* stream) {
    if (!pair_m || !pair_s || !g) return fail(SK_ERR_ARG, "pair_m, pair_s and g must be non-NULL");
    if (B <= 0 || N <= 0 || M <= 0) return fail(SK_ERR_ARG, "bad B, N or M");
    if (!(epsilon > 0.0)) return fail(SK_ERR_ARG, "epsilon must be positive");
    const SolveWs w = carve_solve(workspace, B, N, M);
    if (!workspace || workspace_bytes < w.bytes)
        return fail(SK_ERR_WORKSPACE, "workspace smaller than sk_forward_workspace_bytes");
    const Scalars sc = make_scalars(epsilon, INFINITY, tau_b);
    return launch_col_finish_pairs(pair_m, pair_s, B, M, mask_b, w.log_b, g, w.g_eff, sc,
                                   w.status, (cudaStream_t)stream);
}

int sk_solver_decide(void* workspace, void* stream) {
    if (!workspace) return fail(SK_ERR_ARG, "workspace is NULL");
    launch_pdl(k_decide, dim3(1), dim3(32), 0, (cudaStream_t)stream, (Status*)workspace);
    SK_LAUNCHED("k_decide launch");
    return SK_OK;
}

}  // extern "C"
