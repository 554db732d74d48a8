// sk_fused_kernel.cuh -- one Sinkhorn iteration with a single read of C, on
// clusters of 2, 4 or 8 CTAs; as one step (sk_fused.cu) or as a whole
// persistent solve (sk_fused_solve.cu).
//
// f_new_i depends only on row i of C (and the previous g), so a row can be
// consumed twice while it sits in shared memory: first for its row LSE (the
// f-update), then -- with the f_new just computed -- for the column LSEs of the
// g-update. A cluster of CL CTAs (one per SM) owns a chunk of rows; CTA q owns
// columns [q M/CL, (q+1) M/CL), at most 8192 of them (one 32 KB ring stage),
// so rows of up to 65536 columns stream with one read. Inside a CTA every
// warp has one role and runs its own loop over the chunk's rows; roles meet
// only on mbarriers, so no warp ever waits on a whole group:
//   * producer warp: one cp.async.bulk per row part (rows are contiguous and
//     16-byte aligned) into a kFzStages-deep shared-memory ring;
//   * 8 row warps: each lane reduces its columns of the row part (32 at
//     8192 columns per CTA) to a (max, sum exp) pair in one pass against the
//     previous row's max, with no cross-lane step (slot mbarrier, 8 arrivals);
//   * sender warp: merges the 256 lane pairs into the CTA's pair for the row,
//     stores it locally and into each peer CTA (st.async completing 8 bytes on
//     the peer's slot mbarrier: no cluster-scope fence on the per-row path);
//   * finisher warp: once all CL pairs of row i are present, merges them in
//     rank order (every CTA of the cluster computes the same f_i bit for bit),
//     applies the f-update and posts f_i (slot mbarrier);
//   * 8 column warps: fold row i with f_i into per-column running (reference,
//     sum) states held in registers (one exp per element).
// A stage returns to the producer when all 16 row and column warps are done
// with it. Row slots are indexed modulo kFzSlots > 2 x kFzStages, so neither
// this CTA's warps nor a peer's sender can lap a slot still in use. At the
// end of a chunk's rows each CTA writes one partial column LSE per column.
//
// Step (PERSIST = false): one f-update plus the chunk partials; k_col_finish
// (sk_shard.cu) merges the chunks, applies the g-update, residual and check
// -- or a row-sharded driver exchanges the partials between ranks first.
//
// Solve (PERSIST = true): the whole forward solve in one cooperative launch
// whose clusters are all resident. After each iteration's rows, the warps
// other than the producer meet at a bounded grid barrier, every CTA merges
// the chunk partials of its share of the columns (sk_merge.cuh: the order of
// k_col_finish, so the result is bit-identical to the step path), applies the
// g-update and the residual, meets the others at a second barrier, and reads
// the same residual, so every CTA takes the same convergence decision. The
// producer never joins the barriers: it keeps filling the ring with the next
// iteration's rows meanwhile (C does not change). Data written during the
// launch (g, the partials) is read through L2 only (ld.global.cg).
// Gauss-Seidel order is that of src/sinkhorn/triton/forward.py:161-184; only
// the summation order differs. The check of forward.py:176-182 is the max
// over the whole batch.
//
// Every wait is bounded. A wait that gives up (or sees the abort flag) stops
// its warp and raises this CTA's abort flag, which every other wait polls;
// the last thread out raises the peers' flags and the status's error word,
// which the grid barriers poll. The producer lets its copies land, and all
// CTAs of a cluster meet at the final cluster barrier, so no path can hang or
// leave a CTA's shared memory reachable after it exits.
#pragma once

#include <cmath>
#include <type_traits>

#include "sk_cluster.cuh"
#include "sk_grid.cuh"
#include "sk_merge.cuh"
#include "sk_solve.cuh"
#include "sk_tma.cuh"

namespace sk {

constexpr int kFzRowWarps = 8;    // warps 0-7
constexpr int kFzColWarps = 8;    // warps 8-15
constexpr int kFzProducer = 16;   // warp index of the producer
constexpr int kFzSender = 17;
constexpr int kFzFinisher = 18;
constexpr int kFzThreads = 19 * 32;
constexpr int kFzGroup = kFzRowWarps * 32;     // row lanes covering one row part
constexpr int kFzColLanes = kFzColWarps * 32;  // column lanes covering one row part
constexpr int kFzStages = 6;
constexpr int kFzSlots = 16;      // row slots, > 2 * kFzStages - 2
constexpr int kFzMaxPart = 8192;  // columns per CTA
constexpr int kFzSyncThreads = 18 * 32;   // solve mode: every warp but the producer
constexpr int kFzBarSync = 1;             // their named barrier
constexpr int kFzBarMerge = 2;            // named barrier of the 16 merge warps
constexpr int kFzMergeThreads = 16 * 32;
constexpr uint32_t kFzGridPolls = 1u << 24;

// Rows per chunk: their previous f sits in shared memory (more on the larger
// clusters, whose few clusters each take more rows).
template <int CL>
constexpr int fz_max_rows() {
    return CL <= 2 ? 2048 : 4096;
}

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
    float k2;  // log2(e) / eps, rounded once: the kernel works in log2 units
    float eps, rho, omr;
    Status* st;
    float* lse_out;         // (B,N) the rows' LSE (natural log; -inf masked), or nullptr
    int guard;              // 1: an infinite softmin becomes 0 (the forward's guard)
    // solve mode only: the g-update of the merge and the grid barrier
    float* g;               // (B,M) in place
    float* g_eff_out;       // (B,M) the same buffer as g_eff
    const float* log_b;     // (B,M)
    const uint8_t* mask_b;  // (B,M) or nullptr
    float rho_b, omr_b;
    unsigned* bar;          // grid-barrier arrival counter, zero at launch
};

// A column's running sum is kept relative to a reference that only moves when
// a term would exceed it by more than 2^kLazy, so each term is at most 2^64
// and a chunk's sum stays far inside the fp32 range (2^128) for any chunk
// below 2^60 rows. Terms are flushed only below 2^-126 of the reference,
// which is never above the true column maximum.
constexpr float kLazy = 64.f;
// A row whose terms provably stay below 2^kFastBound of every column reference
// takes the unchecked fold: sums stay below 2^(kFastBound + 24) for chunks of
// up to 2^24 rows, inside the fp32 range.
constexpr float kFastBound = 96.f;
// fp32 C: the column lanes fold the row lanes' exponentials e = 2^(x - lm)
// (x = (g - c) k2, lm the row lane's max), since the column term is
// 2^((f - c) k2) = e * 2^(lm + f k2) * 2^(-g k2): acc = sum of e * 2^(lm +
// f k2 - H) against a per-lane pivot H that moves (rescaling acc) when a
// row's lm + f k2 lies more than kPivotLazy above it, and the column's LSE is
// H + log2(acc) - g k2. A term lost to flushing is below 2^-118 of 2^H, a
// chunk's (at most 2^12 rows) below 2^-106; a column whose sum ends below
// kStarved of 2^H is summed again straight from C.
constexpr float kPivotLazy = 8.f;
constexpr float kStarved = 0x1p-72f;

// Shared-memory layout of k_fused_iter after the ring.
template <int CL>
struct FusedShared {
    uint64_t full[kFzStages];        // stage landed (producer's transaction count)
    uint64_t empty[kFzStages];       // stage free: 8 row + 8 column warps
    uint64_t wpair_bar[kFzSlots];    // the row's 256 lane pairs posted (8 warp arrivals)
    uint64_t hpair_bar[kFzSlots];    // all CL pairs present: local arrive + (CL-1) x 8 bytes
    uint64_t f_bar[kFzSlots];        // f of the row posted
    float2 hpair[kFzSlots][CL];      // [cluster rank]: the CTAs' pairs of a row
    float fq[kFzSlots];              // effective f (-inf for a masked row)
    // per row in the ring: each row lane's (max of x = (g - c) k2, sum of
    // 2^(x - max)); the max also bounds the column lane's terms of that row.
    // The solve mode's merge reuses the space between iterations.
    float2 lpair[kFzStages][kFzGroup];
    float fin[fz_max_rows<CL>()];    // the chunk's previous f, read before any CTA writes f
};

// Loop constants of a solve, in shared memory (no registers across the rows).
struct FzRun {
    int it0, check_every, max_iters;
    float threshold;
};

// (max, sum) pairs in log2 units: sum of 2^(x - max).
__device__ __forceinline__ void lse_merge2(float& m, float& s, float m2, float s2) {
    const float mn = fmaxf(m, m2);
    if (mn == -INFINITY) return;
    s = s * ex2(m - mn) + s2 * ex2(m2 - mn);
    m = mn;
}

// softmin = -eps * LSE in natural units, from a log2-unit pair (with the
// guard of the reference: an infinite softmin becomes 0; an empty row gives
// 0 either way).
__device__ __forceinline__ float softmin_from_pair2(float m, float s, float eps,
                                                    bool guard = true) {
    if (m == -INFINITY) return 0.f;
    float sm = -eps * (kLn2 * (m + log2f(s)));
    if (guard && isinf(sm)) sm = 0.f;
    return sm;
}

// natural-unit LSE of a column state (reference cm, sum cs in log2 units)
__device__ __forceinline__ float lse_nat(float cm, float cs) {
    return cs > 0.f ? kLn2 * (cm + log2f(cs)) : -INFINITY;
}

// Vector g loads: the read-only path in a step (g was written by an earlier
// launch), L2 only in a solve (g is rewritten every iteration of the launch).
template <bool CG>
__device__ __forceinline__ float4 ld_g4(const float* p) {
    if constexpr (CG) return __ldcg(reinterpret_cast<const float4*>(p));
    else return ld_vec4(p);
}

// Row lane t of a staged row part: float4 groups t + 256 u, x = (g - c) k2
// (g - c as fma(c, -1, g), then * k2; column pairs on the packed fp32x2 pipe).
// One pass over the lane's columns in registers: its max lm of x, then the
// sum ls of e = 2^(x - lm). With STORE the exponentials replace the lane's
// elements of C in the ring, where the column lanes fold them. A lane without
// a finite term has ls = 0, or NaN when one of its costs is NaN (a NaN cost
// still reaches f).
template <int G4, bool STORE, typename T>
__device__ __forceinline__ float2 row_lane_exp(T* row, int t, const float (&gk)[4 * G4],
                                               const bool (&gv)[G4], float k2) {
    float2 x[G4][2];
    float m0 = -INFINITY, m1 = -INFINITY;
    const float2 kk = make_float2(k2, k2), neg1 = make_float2(-1.f, -1.f);
#pragma unroll
    for (int u = 0; u < G4; ++u) {
        x[u][0] = x[u][1] = make_float2(-INFINITY, -INFINITY);
        if (!gv[u]) continue;
        const float4 c = lds_c4<T>(row + (t + kFzGroup * u) * 4);
        x[u][0] = __fmul2_rn(
            __ffma2_rn(make_float2(c.x, c.y), neg1, make_float2(gk[4 * u + 0], gk[4 * u + 1])),
            kk);
        x[u][1] = __fmul2_rn(
            __ffma2_rn(make_float2(c.z, c.w), neg1, make_float2(gk[4 * u + 2], gk[4 * u + 3])),
            kk);
        m0 = fmaxf(m0, fmaxf(x[u][0].x, x[u][0].y));
        m1 = fmaxf(m1, fmaxf(x[u][1].x, x[u][1].y));
    }
    const float lm = fmaxf(m0, m1);
    if (lm == -INFINITY) {
        bool nan = false;
#pragma unroll
        for (int u = 0; u < G4; ++u) {
            nan = nan || isnan(x[u][0].x) || isnan(x[u][0].y) || isnan(x[u][1].x) ||
                  isnan(x[u][1].y);
            if constexpr (STORE)
                if (gv[u])
                    *reinterpret_cast<float4*>(row + (t + kFzGroup * u) * 4) =
                        make_float4(0.f, 0.f, 0.f, 0.f);
        }
        return make_float2(lm, nan ? NAN : 0.f);
    }
    const float2 nm = make_float2(-lm, -lm);
    float2 s01 = make_float2(0.f, 0.f), s23 = s01;
#pragma unroll
    for (int u = 0; u < G4; ++u) {
        if (!gv[u]) continue;
        const float2 d01 = __fadd2_rn(x[u][0], nm), d23 = __fadd2_rn(x[u][1], nm);
        const float2 e01 = make_float2(ex2(d01.x), ex2(d01.y));
        const float2 e23 = make_float2(ex2(d23.x), ex2(d23.y));
        s01 = __fadd2_rn(s01, e01);
        s23 = __fadd2_rn(s23, e23);
        if constexpr (STORE)
            *reinterpret_cast<float4*>(row + (t + kFzGroup * u) * 4) =
                make_float4(e01.x, e01.y, e23.x, e23.y);
    }
    return make_float2(lm, (s01.x + s01.y) + (s23.x + s23.y));
}

// Column j's LSE (log2 units) over the chunk's rows straight from C, with the
// rows' new f (fn, 0 at masked rows) and a running max: the fold of a column
// whose pivoted sum ended below kStarved.
static __device__ __noinline__ float fz_column_direct(const float* Cj, int64_t sCn, const float* fn,
                                               const uint8_t* mask, uint32_t rows, float k2) {
    float m = -INFINITY, s = 0.f;
    for (uint32_t i = 0; i < rows; ++i) {
        if (mask != nullptr && mask[i] == 0) continue;
        const float y = (fn[i] - Cj[(int64_t)i * sCn]) * k2;
        if (y > m) {
            s = s * ex2(m - y) + 1.f;
            m = y;
        } else if (y == y) {
            s += ex2(y - m);
        } else {
            m = y;  // NaN
        }
    }
    return m == -INFINITY ? -INFINITY : m + log2f(s);
}

// The end of one iteration of a solve, for the 18 warps other than the
// producer (one copy of the code, called by every role): grid barrier (all
// chunk partials written), merge of this CTA's 32-column tiles with the
// g-update and g residual (warps 0-15: tile slot w / 4, merge subset w % 4;
// tiles blockIdx + (4 r + slot) gridDim), grid barrier (g complete), and the
// convergence decision taken from the one residual every CTA reads. Returns
// true to run the next iteration. sa: the kernel arguments in shared memory.
static __device__ __noinline__ bool fz_end_iteration(const FusedArgs& sa, const FzRun& run,
                                              float2* mp_base, volatile int* flag, int* sh_ok,
                                              int* sh_done, int it) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool leader = threadIdx.x == 0;
    Status* st = sa.st;
    unsigned* err_word = reinterpret_cast<unsigned*>(&st->err);
    const int64_t BM = sa.B * sa.M;
    const int itg = run.it0 + it;
    const bool check = run.check_every > 0 && (itg + 1) % run.check_every == 0;
    const int kc = check ? (itg + 1) / run.check_every - 1 : 0;
    named_bar_sync(kFzBarSync, kFzSyncThreads);
    if (leader) {
        const bool ok = *flag == 0 && grid_sync_counter(sa.bar, (unsigned)(2 * it + 1) * gridDim.x,
                                                        err_word, kFzGridPolls);
        if (!ok) {
            *flag = 1;
            atomicMax(&st->err, 2);
        }
        *sh_ok = ok ? 1 : 0;
    }
    named_bar_sync(kFzBarSync, kFzSyncThreads);
    if (!*sh_ok) return false;
    if (warp < kFzRowWarps + kFzColWarps) {
        const int j = warp >> 2, sub = warp & 3;
        float2(*mp)[kMergeSubsets][32] = reinterpret_cast<float2(*)[kMergeSubsets][32]>(mp_base);
        const int64_t ntile = (BM + 31) / 32;
        const int64_t G = gridDim.x;
        const int64_t rounds = (ntile + 4 * G - 1) / (4 * G);
        const int64_t ps = BM + 4;
        for (int64_t r = 0; r < rounds; ++r) {
            const int64_t t = (int64_t)blockIdx.x + (4 * r + j) * G;
            const int64_t col = t * 32 + lane;
            const bool live = col < BM;
            mp[j][sub][lane] = merge_subset<true>(sa.parts + col, ps, (int)sa.chunks, sub, live);
            named_bar_sync(kFzBarMerge, kFzMergeThreads);
            if (sub == 0) {
                float res = 0.f;
                if (live) {
                    const float2 sp[kMergeSubsets] = {mp[j][0][lane], mp[j][1][lane],
                                                      mp[j][2][lane], mp[j][3][lane]};
                    float mm, ss;
                    merge_subsets(mm, ss, sp);
                    const float gin = __ldcg(sa.g + col);
                    const bool valid = (sa.mask_b == nullptr) || (sa.mask_b[col] != 0);
                    float go = 0.f;  // masked_fill(~mask_b, 0)
                    if (valid) {
                        const float full = softmin_from_pair(mm, ss, sa.eps, true) +
                                           sa.eps * __ldg(sa.log_b + col);
                        go = (sa.rho_b == 0.f) ? full : sa.rho_b * gin + sa.omr_b * full;
                    }
                    sa.g[col] = go;
                    sa.g_eff_out[col] = valid ? go : -INFINITY;
                    res = fabsf(go - gin);
                }
                if (check) {
                    float rr = warp_max(res);
                    if (__any_sync(0xffffffffu, isnan(res))) rr = NAN;
                    if (lane == 0) atomic_max_nonneg(&st->res_slot[kc % 3], rr);
                }
            }
            named_bar_sync(kFzBarMerge, kFzMergeThreads);
        }
    }
    named_bar_sync(kFzBarSync, kFzSyncThreads);
    if (leader) {
        const bool ok = grid_sync_counter(sa.bar, (unsigned)(2 * it + 2) * gridDim.x, err_word,
                                          kFzGridPolls);
        int done = 0;
        if (ok) {
            unsigned rb = 0u;
            if (check) rb = atomicOr(&st->res_slot[kc % 3], 0u);
            const bool conv = check && __uint_as_float(rb) < run.threshold;
            done = (conv || itg + 1 >= run.max_iters) ? 1 : 0;
            if (check && blockIdx.x == 0) {
                // the slot of the check after next: every reader of its last
                // use has passed this barrier and no writer has reached it
                st->res_slot[(kc + 2) % 3] = 0u;
                st->res_bits = rb;
            }
            if (done && blockIdx.x == 0) {
                st->converged = conv ? 1 : 0;
                st->n_iters = itg + 1;
                st->iter = itg + 1;
                st->done = 1;
            }
        } else {
            *flag = 1;
            atomicMax(&st->err, 2);
        }
        *sh_ok = ok ? 1 : 0;
        *sh_done = done;
        if (done) *flag = 2;  // the producer stops refilling the ring
    }
    named_bar_sync(kFzBarSync, kFzSyncThreads);
    return *sh_ok && !*sh_done;
}

// G4 = float4 column groups per thread within the CTA's row part; FULL: the
// part is exactly kFzGroup * 4 * G4 columns (no bounds guards).
// 19 warps: one SM sub-partition holds 5 of them, so 16,384 / (5 x 32) caps
// a thread at 96 registers (one CTA per SM).
// T: element type of C (float, or uint16_t holding bf16); the ring holds T.
template <int G4, bool FULL, int CL, bool PERSIST, typename T = float>
__global__ void __cluster_dims__(CL, 1, 1) __launch_bounds__(kFzThreads, 1)
    k_fused_iter(FusedArgs a) {
    pdl_wait();
    if constexpr (!PERSIST) pdl_trigger();
    constexpr int NV = 4 * G4;  // columns per thread
    constexpr int kMaxRows = fz_max_rows<CL>();
    extern __shared__ __align__(128) unsigned char smem[];
    const int64_t part = a.M / CL;
    T* ring = reinterpret_cast<T*>(smem);
    FusedShared<CL>& S =
        *reinterpret_cast<FusedShared<CL>*>(smem + (size_t)kFzStages * part * sizeof(T));
    __shared__ volatile int sh_abort;  // 0 running, 1 abort, 2 stop (solve done)
    __shared__ int sh_ok, sh_done;
    __shared__ FzRun run;
    __shared__ FusedArgs sa;  // solve mode: the arguments for fz_end_iteration

    Status* st = a.st;
    if (read_volatile(&st->done)) return;  // every CTA of the grid reads the same flag
    const int iter0 = read_volatile(&st->iter);
    const bool check = is_check_iter(st, iter0);  // (a step's check)
    // iterations of this launch
    const int n_run = PERSIST ? max(st->max_iters - iter0, 0) : 1;
    const uint32_t rank = cluster_ctarank();
    const int64_t unit = blockIdx.x / CL;
    const int64_t b = unit / a.chunks;
    const int64_t chunk = unit - b * a.chunks;
    const int64_t r0 = chunk * a.rows_per_chunk;
    const int64_t r1 = (r0 + a.rows_per_chunk) < a.N ? (r0 + a.rows_per_chunk) : a.N;
    const int64_t R = r1 > r0 ? r1 - r0 : 0;  // <= kMaxRows: the row loops count in 32 bits
    const int64_t col0 = (int64_t)rank * part;
    if (a.rows_per_chunk > kMaxRows || n_run == 0) {  // the plan never does this; uniform
        if (threadIdx.x == 0 && blockIdx.x == 0 && n_run > 0) atomicMax(&st->err, 3);
        return;
    }
    // f is updated in place and every CTA of a row needs its previous value:
    // copy it before the cluster barrier below, after which rank 0 writes f
    for (int64_t r = threadIdx.x; r < R; r += kFzThreads) S.fin[r] = a.f_in[b * a.N + r0 + r];

    if (threadIdx.x == 0) {
        for (int q = 0; q < kFzStages; ++q) {
            mbar_init(&S.full[q], 1);
            mbar_init(&S.empty[q], kFzRowWarps + kFzColWarps);
        }
        for (int q = 0; q < kFzSlots; ++q) {
            mbar_init(&S.wpair_bar[q], kFzRowWarps);
            mbar_init(&S.hpair_bar[q], 1);
            mbar_init(&S.f_bar[q], 1);
        }
        sh_abort = 0;
        if constexpr (PERSIST) {
            sh_done = 0;
            run.it0 = iter0;
            run.check_every = st->check_every;
            run.max_iters = st->max_iters;
            run.threshold = st->threshold;
            sa = a;
        }
        mbar_init_fence();
    }
    __syncthreads();
    __syncwarp();
    cluster_barrier();  // the peers' barriers exist before any remote arrive

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rows = (uint32_t)R;
    if (warp == kFzProducer) {
        // ---- producer: one bulk copy of the row part per stage -----------
        if (lane == 0 && R > 0) {
            const T* src = reinterpret_cast<const T*>(a.C) + b * a.sCb + r0 * a.sCn + col0;
            const uint32_t bytes = (uint32_t)(part * sizeof(T));
            uint32_t issued = 0;
            bool stopped = false;
            for (int it = 0; it < n_run && !stopped; ++it) {
                for (uint32_t i = 0; i < rows; ++i) {
                    const uint32_t s = (uint32_t)it * rows + i;  // stage sequence number
                    const int q = (int)(s % kFzStages);
                    if (s >= kFzStages &&
                        !wait_full(&S.empty[q], ((s / kFzStages) - 1) & 1u, &sh_abort)) {
                        stopped = true;
                        break;
                    }
                    mbar_expect_tx(&S.full[q], bytes);
                    bulk_g2s(ring + (size_t)q * part, src + (int64_t)i * a.sCn, bytes,
                             &S.full[q]);
                    issued = s + 1;
                }
            }
            if (stopped && sh_abort == 0) sh_abort = 1;  // a wait ran out
            // every issued copy lands before the CTA can leave (bounded)
            const uint32_t first = issued > kFzStages ? issued - kFzStages : 0;
            for (uint32_t s = first; s < issued; ++s)
                if (!mbar_wait(&S.full[s % kFzStages], (s / kFzStages) & 1u)) sh_abort = 1;
        }
        __syncwarp();
    } else if (warp < kFzRowWarps) {
        // ---- row warp: (max, sum exp) of its slice of each row part -------
        const int t = threadIdx.x;
        const float k2 = a.k2;
        bool gv[G4];
#pragma unroll
        for (int u = 0; u < G4; ++u) gv[u] = FULL || (int64_t)(t + kFzGroup * u) * 4 < part;
        for (int it = 0; it < n_run; ++it) {
            bool ok = true;
            float gk[NV];
#pragma unroll
            for (int u = 0; u < G4; ++u) {
                float4 g4 = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
                if (gv[u]) g4 = ld_g4<PERSIST>(a.g_eff + b * a.M + col0 + (t + kFzGroup * u) * 4);
                gk[4 * u + 0] = g4.x;
                gk[4 * u + 1] = g4.y;
                gk[4 * u + 2] = g4.z;
                gk[4 * u + 3] = g4.w;
            }
            for (uint32_t i = 0; i < rows; ++i) {
                const uint32_t s = (uint32_t)it * rows + i;
                const int q = (int)(s % kFzStages);
                if (!warp_wait(&S.full[q], (uint32_t)(s / kFzStages) & 1u, &sh_abort)) {
                    if (lane == 0 && sh_abort == 0) sh_abort = 1;
                    ok = false;
                    break;
                }
                T* row = ring + (size_t)q * part;
                // fp32 C: the exponentials replace this lane's costs in the stage
                const float2 pr = row_lane_exp<G4, std::is_same<T, float>::value>(row, t, gk, gv, k2);
                S.lpair[q][t] = pr;
                __syncwarp();  // every lane's stores precede the arrives
                if (lane == 0) {
                    mbar_arrive(&S.empty[q]);  // this warp is done with the stage
                    mbar_arrive(&S.wpair_bar[(int)(s % kFzSlots)]);
                }
            }
            if constexpr (PERSIST) {
                if (!fz_end_iteration(sa, run, &S.lpair[0][0], &sh_abort, &sh_ok, &sh_done, it) ||
                    !ok)
                    break;
            }
        }
    } else if (warp == kFzSender) {
        // ---- sender: this CTA's pair of the row, to itself and the peers ---
        uint32_t remote_pair0[CL > 1 ? CL - 1 : 1], remote_bar0[CL > 1 ? CL - 1 : 1];
#pragma unroll
        for (int p = 0; p < CL - 1; ++p) {
            const uint32_t peer = (uint32_t)p < rank ? (uint32_t)p : (uint32_t)p + 1u;
            remote_pair0[p] = map_to_rank(&S.hpair[0][rank], peer);
            remote_bar0[p] = map_to_rank(&S.hpair_bar[0], peer);
        }
        for (int it = 0; it < n_run; ++it) {
            bool ok = true;
            for (uint32_t i = 0; i < rows; ++i) {
                const uint32_t s = (uint32_t)it * rows + i;
                const int sl = (int)(s % kFzSlots);
                if (!warp_wait(&S.wpair_bar[sl], (uint32_t)(s / kFzSlots) & 1u, &sh_abort)) {
                    if (lane == 0 && sh_abort == 0) sh_abort = 1;
                    ok = false;
                    break;
                }
                // 256 lane pairs: their max, then the rescaled sum
                const int q = (int)(s % kFzStages);
                constexpr int kPer = kFzGroup / 32;
                float pm[kPer], ps[kPer];
                float m = -INFINITY;
#pragma unroll
                for (int k = 0; k < kPer; ++k) {
                    const float2 p = S.lpair[q][lane + 32 * k];
                    pm[k] = p.x;
                    ps[k] = p.y;
                    m = fmaxf(m, p.x);
                }
                m = warp_max(m);
                float sum = 0.f;
#pragma unroll
                for (int k = 0; k < kPer; ++k)  // (an all-empty row sums its 0 / NaN lanes)
                    sum = m == -INFINITY ? sum + ps[k] : fmaf(ps[k], ex2(pm[k] - m), sum);
                sum = warp_sum(sum);
                if (lane == 0) {
                    S.hpair[sl][rank] = make_float2(m, sum);
#pragma unroll
                    for (int p = 0; p < CL - 1; ++p)
                        st_async_f32x2(remote_pair0[p] + (uint32_t)(sl * CL) * sizeof(float2),
                                       m, sum, remote_bar0[p] + (uint32_t)sl * sizeof(uint64_t));
                    // this CTA's arrival; the phase also waits for the peers' bytes
                    mbar_expect_tx(&S.hpair_bar[sl], (uint32_t)((CL - 1) * sizeof(float2)));
                }
                __syncwarp();
            }
            if constexpr (PERSIST) {
                if (!fz_end_iteration(sa, run, &S.lpair[0][0], &sh_abort, &sh_ok, &sh_done, it) ||
                    !ok)
                    break;
            }
        }
    } else if (warp == kFzFinisher) {
        // ---- finisher: f_i from all CTAs' pairs -----------------------------
        for (int it = 0; it < n_run; ++it) {
            bool ok = true;
            bool chk = check;
            int kc = 0;
            if constexpr (PERSIST) {
                const int itg = run.it0 + it;
                chk = run.check_every > 0 && (itg + 1) % run.check_every == 0;
                kc = chk ? (itg + 1) / run.check_every - 1 : 0;
            }
            float res = 0.f;
            // the rows' log a and mask, 32 rows per block: lane k holds row
            // 32 j + k of block j, and block j + 1 is loaded while block j is
            // in use, so no row waits for its scalars
            auto blk_load = [&](uint32_t j, float& la, int& vk) {
                const uint32_t r = 32u * j + (uint32_t)lane;
                la = 0.f;
                vk = 0;
                if (r < rows) {
                    const int64_t g = b * a.N + r0 + r;
                    la = __ldg(a.log_a + g);
                    vk = (a.mask_a == nullptr || a.mask_a[g] != 0) ? 1 : 0;
                }
            };
            float la_cur, la_nxt;
            int vk_cur, vk_nxt;
            blk_load(0u, la_cur, vk_cur);
            blk_load(1u, la_nxt, vk_nxt);
            for (uint32_t i = 0; i < rows; ++i) {
                if (i > 0 && (i & 31u) == 0) {
                    la_cur = la_nxt;
                    vk_cur = vk_nxt;
                    blk_load(i / 32u + 1u, la_nxt, vk_nxt);
                }
                const float lav = __shfl_sync(0xffffffffu, la_cur, (int)(i & 31u));
                const bool valid = __shfl_sync(0xffffffffu, vk_cur, (int)(i & 31u)) != 0;
                const uint32_t s = (uint32_t)it * rows + i;
                const int sl = (int)(s % kFzSlots);
                if (!warp_wait_peer(&S.hpair_bar[sl], (uint32_t)(s / kFzSlots) & 1u,
                                    &sh_abort)) {
                    if (lane == 0 && sh_abort == 0) sh_abort = 1;
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    const float fin = S.fin[i];
                    float mm = S.hpair[sl][0].x, ss = S.hpair[sl][0].y;
#pragma unroll
                    for (int p = 1; p < CL; ++p)  // rank order: identical in every CTA
                        lse_merge2(mm, ss, S.hpair[sl][p].x, S.hpair[sl][p].y);
                    float fo = 0.f;  // masked_fill(~mask_a, 0)
                    if (valid) {
                        const float sm = softmin_from_pair2(mm, ss, a.eps, a.guard != 0);
                        const float fullv = sm + a.eps * lav;
                        fo = (a.rho == 0.f) ? fullv : a.rho * fin + a.omr * fullv;
                    }
                    const float fe = valid ? fo : -INFINITY;
                    S.fq[sl] = fe;
                    mbar_arrive(&S.f_bar[sl]);
                    // the new f: the next iteration's previous f (solve mode) and
                    // the direct fold of a starved column
                    S.fin[i] = fo;
                    if (rank == 0) {
                        const int64_t grow = b * a.N + r0 + i;
                        a.f_out[grow] = fo;
                        a.f_eff[grow] = fe;
                        if (a.lse_out)
                            a.lse_out[grow] = (valid && mm != -INFINITY)
                                                  ? kLn2 * (mm + log2f(ss)) : -INFINITY;
                        const float d = fabsf(fo - fin);
                        res = (d > res || isnan(d)) ? d : res;
                    }
                }
                __syncwarp();
            }
            if (lane == 0 && rank == 0) {
                if constexpr (PERSIST) {
                    if (chk) atomic_max_nonneg(&st->res_slot[kc % 3], res);
                } else {
                    if (b == 0) a.parts[chunk * (a.B * a.M + 4) + a.B * a.M] = 0.f;
                    if (chk) atomic_max_nonneg(&st->res_bits, res);
                }
            }
            __syncwarp();
            if constexpr (PERSIST) {
                if (!fz_end_iteration(sa, run, &S.lpair[0][0], &sh_abort, &sh_ok, &sh_done, it) ||
                    !ok)
                    break;
            }
        }
    } else if constexpr (std::is_same<T, float>::value) {
        // ---- column warp: fold the row lanes' exponentials with f_i -------
        // column lane tc holds float4 groups tc + 256 u of the row part, the
        // columns of row lane tc, whose (max, sum) pair gives its row factor
        const int tc = threadIdx.x - kFzGroup;
        const float k2 = a.k2;
        bool gv[G4];
#pragma unroll
        for (int u = 0; u < G4; ++u) gv[u] = FULL || (int64_t)(tc + kFzColLanes * u) * 4 < part;
        const float* gsrc = a.g_eff + b * a.M + col0;
        for (int it = 0; it < n_run; ++it) {
            bool ok = true;
            float2 acc[G4][2];
#pragma unroll
            for (int u = 0; u < G4; ++u) acc[u][0] = acc[u][1] = make_float2(0.f, 0.f);
            float H = -INFINITY;  // this lane's pivot (log2 units)
            for (uint32_t i = 0; i < rows; ++i) {
                const uint32_t s = (uint32_t)it * rows + i;
                const int sl = (int)(s % kFzSlots);
                if (!warp_wait(&S.f_bar[sl], (uint32_t)(s / kFzSlots) & 1u, &sh_abort)) {
                    if (lane == 0 && sh_abort == 0) sh_abort = 1;
                    ok = false;
                    break;
                }
                const float f = S.fq[sl];
                const int q = (int)(s % kFzStages);
                const float lm = S.lpair[q][tc].x;
                // a masked row has no terms; a NaN f reaches every column
                if (f != -INFINITY && (lm != -INFINITY || isnan(f))) {
                    const float rb = lm + f * k2;  // bound of the lane's terms of the row
                    if (!(rb <= H + kPivotLazy)) {
                        const float sc = ex2(H - rb);  // 0 while no row has been folded
                        const float2 sc2 = make_float2(sc, sc);
#pragma unroll
                        for (int u = 0; u < G4; ++u) {
                            acc[u][0] = __fmul2_rn(acc[u][0], sc2);
                            acc[u][1] = __fmul2_rn(acc[u][1], sc2);
                        }
                        H = rb;
                    }
                    const float F = ex2(rb - H);
                    const float2 F2 = make_float2(F, F);
                    const float* row = reinterpret_cast<const float*>(ring) + (size_t)q * part;
#pragma unroll
                    for (int u = 0; u < G4; ++u) {
                        if (!gv[u]) continue;
                        const float4 e = *reinterpret_cast<const float4*>(
                            row + (tc + kFzColLanes * u) * 4);
                        acc[u][0] = __ffma2_rn(make_float2(e.x, e.y), F2, acc[u][0]);
                        acc[u][1] = __ffma2_rn(make_float2(e.z, e.w), F2, acc[u][1]);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.empty[q]);
            }
            // this chunk's column partials (natural-log LSE per column)
            if (ok) {
                const int64_t pstride = a.B * a.M + 4;  // keeps every chunk row 16-byte aligned
                float* dst = a.parts + chunk * pstride + b * a.M + col0;
                const uint8_t* mrow = a.mask_a == nullptr ? nullptr : a.mask_a + b * a.N + r0;
#pragma unroll
                for (int u = 0; u < G4; ++u) {
                    if (!gv[u]) continue;
                    const int64_t c4 = (int64_t)(tc + kFzColLanes * u) * 4;
                    const float4 g4 = ld_g4<PERSIST>(gsrc + c4);
                    const float gg[4] = {g4.x, g4.y, g4.z, g4.w};
                    const float av[4] = {acc[u][0].x, acc[u][0].y, acc[u][1].x, acc[u][1].y};
                    float o[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        o[e] = -INFINITY;  // a masked column, or no valid row in the chunk
                        if (gg[e] != -INFINITY && H != -INFINITY) {
                            if (!(av[e] < kStarved))
                                o[e] = kLn2 * (H + log2f(av[e]) - gg[e] * k2);
                            else
                                o[e] = kLn2 * fz_column_direct(
                                                  reinterpret_cast<const float*>(a.C) + b * a.sCb +
                                                      r0 * a.sCn + col0 + c4 + e,
                                                  a.sCn, S.fin, mrow, rows, k2);
                        }
                    }
                    *reinterpret_cast<float4*>(dst + c4) = make_float4(o[0], o[1], o[2], o[3]);
                }
            }
            if constexpr (PERSIST) {
                if (!fz_end_iteration(sa, run, &S.lpair[0][0], &sh_abort, &sh_ok, &sh_done, it) ||
                    !ok)
                    break;
            }
        }
    } else {
        // ---- column warp: fold row i with f_i into the column states -----
        // column lane tc holds float4 groups tc + 256 u of the row part, the
        // columns of row lane tc (whose max bounds their terms)
        constexpr int CG4 = G4;
        constexpr int CNV = 4 * CG4;
        const int tc = threadIdx.x - kFzGroup;
        const int tr = tc & (kFzGroup - 1);
        const float k2 = a.k2;
        bool gv[CG4];
#pragma unroll
        for (int u = 0; u < CG4; ++u)
            gv[u] = FULL || (int64_t)(tc + kFzColLanes * u) * 4 < part;
        const float* gsrc = a.g_eff + b * a.M + col0;
        for (int it = 0; it < n_run; ++it) {
            bool ok = true;
            float cm[CNV], cs[CNV];  // per column: reference (log2 units) and sum of 2^(y - cm)
#pragma unroll
            for (int v = 0; v < CNV; ++v) {
                cm[v] = -3.0e38f;  // finite start: an empty column keeps cs = 0
                cs[v] = 0.f;
            }
            // hmin = min over this lane's unmasked columns of g * k2 + cm. Term
            // (f - c) k2 - cm = x + (f - g) k2 - cm <= lmax + f k2 - hmin, with x =
            // (g - c) k2 and lmax row lane tr's max of x over the same columns.
            float hmin = -INFINITY;  // no bound before the first row sets cm
            for (uint32_t i = 0; i < rows; ++i) {
                const uint32_t s = (uint32_t)it * rows + i;
                const int sl = (int)(s % kFzSlots);
                if (!warp_wait(&S.f_bar[sl], (uint32_t)(s / kFzSlots) & 1u, &sh_abort)) {
                    if (lane == 0 && sh_abort == 0) sh_abort = 1;
                    ok = false;
                    break;
                }
                const float f = S.fq[sl];
                const int q = (int)(s % kFzStages);
                const float bound = S.lpair[q][tr].x + f * k2 - hmin;
                if (!warp_wait(&S.full[q], (uint32_t)(s / kFzStages) & 1u, &sh_abort)) {
                    if (lane == 0 && sh_abort == 0) sh_abort = 1;
                    ok = false;
                    break;
                }
                const T* row = ring + (size_t)q * part;
                if (f != -INFINITY) {
                    if (bound <= kFastBound) {
                        // every term is below 2^kFastBound: no per-element check;
                        // column pairs through the packed fp32x2 pipe, rounded as
                        // the scalar (f - c) * k2 - cm
                        const float2 ff = make_float2(f, f), kk = make_float2(k2, k2);
                        const float2 neg1 = make_float2(-1.f, -1.f);
#pragma unroll
                        for (int u = 0; u < CG4; ++u) {
                            if (!gv[u]) continue;
                            const float4 c = lds_c4<T>(row + (tc + kFzColLanes * u) * 4);
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                const int v = 4 * u + 2 * h;
                                const float2 cc =
                                    h ? make_float2(c.z, c.w) : make_float2(c.x, c.y);
                                const float2 y = __fmul2_rn(__ffma2_rn(cc, neg1, ff), kk);
                                const float2 d =
                                    __ffma2_rn(make_float2(cm[v], cm[v + 1]), neg1, y);
                                const float2 sum = __fadd2_rn(make_float2(cs[v], cs[v + 1]),
                                                              make_float2(ex2(d.x), ex2(d.y)));
                                cs[v] = sum.x;
                                cs[v + 1] = sum.y;
                            }
                        }
                    } else {
#pragma unroll
                        for (int u = 0; u < CG4; ++u) {
                            if (!gv[u]) continue;
                            const float4 c = lds_c4<T>(row + (tc + kFzColLanes * u) * 4);
                            const float y[4] = {(f - c.x) * k2, (f - c.y) * k2, (f - c.z) * k2,
                                                (f - c.w) * k2};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                // a term far above its column's reference (and the
                                // first row of every column) moves the reference to it
                                const int v = 4 * u + e;
                                const float d = y[e] - cm[v];
                                if (d > kLazy) {
                                    cs[v] = fmaf(cs[v], ex2(-d), 1.f);
                                    cm[v] = y[e];
                                } else {
                                    cs[v] += ex2(d);
                                }
                            }
                        }
                        // references may have moved: recompute the bound's minimum
                        float h = INFINITY;
#pragma unroll
                        for (int u = 0; u < CG4; ++u) {
                            if (!gv[u]) continue;
                            const float4 g4 = ld_g4<PERSIST>(gsrc + (tc + kFzColLanes * u) * 4);
                            const float gg[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
                            for (int e = 0; e < 4; ++e)
                                if (gg[e] != -INFINITY) h = fminf(h, gg[e] * k2 + cm[4 * u + e]);
                        }
                        hmin = h;
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.empty[q]);
            }
            // this chunk's column partials (natural-log LSE per column)
            if (ok) {
                const int64_t pstride = a.B * a.M + 4;  // keeps every chunk row 16-byte aligned
                float* dst = a.parts + chunk * pstride + b * a.M + col0;
#pragma unroll
                for (int u = 0; u < CG4; ++u) {
                    if (!gv[u]) continue;
                    const int64_t c4 = (int64_t)(tc + kFzColLanes * u) * 4;
                    float4 o;
                    o.x = lse_nat(cm[4 * u + 0], cs[4 * u + 0]);
                    o.y = lse_nat(cm[4 * u + 1], cs[4 * u + 1]);
                    o.z = lse_nat(cm[4 * u + 2], cs[4 * u + 2]);
                    o.w = lse_nat(cm[4 * u + 3], cs[4 * u + 3]);
                    *reinterpret_cast<float4*>(dst + c4) = o;
                }
            }
            if constexpr (PERSIST) {
                if (!fz_end_iteration(sa, run, &S.lpair[0][0], &sh_abort, &sh_ok, &sh_done, it) ||
                    !ok)
                    break;
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0 && sh_abort == 1) {
        atomicMax(&st->err, 2);
        // peers waiting for this CTA's pairs stop at once instead of timing out
#pragma unroll
        for (uint32_t p = 0; p < (uint32_t)CL; ++p)
            if (p != rank) st_cluster_u32(map_to_rank((const void*)&sh_abort, p), 1u);
    }
    __syncwarp();
    cluster_barrier();  // no CTA leaves while a peer may still touch its shared memory
}

// Dynamic shared memory of k_fused_iter for a row part of `part` elements.
template <int CL, typename T>
constexpr size_t fz_smem(int64_t part) {
    return (size_t)kFzStages * (size_t)part * sizeof(T) + sizeof(FusedShared<CL>);
}

// Opt in to more than 48 KB of dynamic shared memory, once per device and
// instantiation.
template <int G4, bool FULL, int CL, bool PERSIST, typename T>
static int fz_prepare() {
    static thread_local unsigned long long ready = 0;  // bit per device ordinal
    int dev = 0;
    SK_CUDA(cudaGetDevice(&dev));
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(ready & bit)) {
        SK_CUDA(cudaFuncSetAttribute(k_fused_iter<G4, FULL, CL, PERSIST, T>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)fz_smem<CL, T>(kFzMaxPart)));
        SK_CUDA(cudaFuncSetAttribute(k_fused_iter<G4, FULL, CL, PERSIST, T>,
                                     cudaFuncAttributePreferredSharedMemoryCarveout,
                                     (int)cudaSharedmemCarveoutMaxShared));
        ready |= bit;
    }
    return SK_OK;
}

// The kernel arguments of a problem's chunking (sk_fused.cu).
FusedArgs fused_args(const Problem& P, const SolveWs& w, const Scalars& sc,
                     const uint8_t* mask_a, float* f, int64_t chunks, int64_t rows_per_chunk);
// Co-resident clusters of cluster size CL on the current device (0: unknown).
int64_t fz_active_clusters(int CL);

// Cluster size of the single-read iteration for rows of M columns (0: none):
// 2 for 2048..16384, 4 up to 32768, 8 up to 65536, with 16-byte row parts.
// (plan_fused runs 2048 < M < 8192 on one-CTA "clusters": a CTA holds the
// whole row and the pair exchange is local.)
inline int fz_cluster_size(int64_t M) {
    if (M >= 2048 && M <= 16384 && M % 8 == 0) return 2;
    if (M > 16384 && M <= 32768 && M % 16 == 0) return 4;
    if (M > 32768 && M <= 65536 && M % 32 == 0) return 8;
    return 0;
}

}  // namespace sk
