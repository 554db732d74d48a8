// sk_fused.cu -- one Sinkhorn iteration with a single read of C.
//
// f_new_i depends only on row i of C (and the previous g), so a row can be
// consumed twice while it sits in shared memory: first for its row LSE (the
// f-update), then -- with the f_new just computed -- for the column LSEs of the
// g-update. A cluster of two CTAs (one per SM) owns a chunk of rows; CTA q
// owns columns [q M/2, (q+1) M/2). Inside a CTA every warp has one role and
// runs its own loop over the chunk's rows; roles meet only on mbarriers, so
// no warp ever waits on a whole group:
//   * producer warp: one cp.async.bulk per half-row (rows are contiguous and
//     16-byte aligned) into a kFzStages-deep shared-memory ring;
//   * 8 row warps: each lane reduces its columns of the half-row (32 at
//     M = 16384) to a (max, sum exp) pair in one pass against the previous
//     row's max, with no cross-lane step (slot mbarrier, 8 arrivals);
//   * sender warp: merges the 256 lane pairs into the half-row pair, stores it
//     locally and into the peer CTA (st.async completing bytes on the peer's
//     slot mbarrier: no cluster-scope fence on the per-row path);
//   * finisher warp: once both halves' pairs of row i are present, merges
//     them in rank order (both CTAs compute the same f_i bit for bit), applies
//     the f-update and posts f_i (slot mbarrier);
//   * 8 column warps: fold row i with f_i into per-column running (reference,
//     sum) states held in registers (one exp per element).
// A stage returns to the producer when all 16 row and column warps are done
// with it. Row slots are indexed modulo kFzSlots > 2 x kFzStages, so neither
// this CTA's warps nor the peer's sender can lap a slot still in use. At the
// end each CTA writes one partial column LSE per column; k_col_finish
// (sk_shard.cu) merges the chunks, applies the g-update, residual and check.
// Gauss-Seidel order is that of src/sinkhorn/triton/forward.py:161-184; only
// the summation order differs.
//
// Every wait is bounded. A wait that gives up (or sees the abort flag) stops
// its warp and raises this CTA's abort flag, which every other wait polls;
// the last thread out raises the peer's flag too. The producer lets its copies
// land, and both CTAs meet at the final cluster barrier, so no path can hang
// or leave a CTA's shared memory reachable after it exits.
#include <algorithm>
#include <cmath>

#include "sk_internal.h"
#include "sk_solve.cuh"
#include "sk_cluster.cuh"
#include "sk_tma.cuh"

namespace sk {

constexpr int kFzRowWarps = 8;    // warps 0-7
constexpr int kFzColWarps = 8;    // warps 8-15
constexpr int kFzProducer = 16;   // warp index of the producer
constexpr int kFzSender = 17;
constexpr int kFzFinisher = 18;
constexpr int kFzThreads = 19 * 32;
constexpr int kFzGroup = kFzRowWarps * 32;     // row lanes covering one half-row
constexpr int kFzColLanes = kFzColWarps * 32;  // column lanes covering one half-row
// A row lane sums 2^(x - ref) against the previous row's max; the pass is kept
// when this row's max lies in [ref - kRefBelow, ref + kRefAbove] (terms stay
// below 2^kRefAbove, and only terms below 2^-66 of the max can flush).
constexpr float kRefAbove = 100.f;
constexpr float kRefBelow = 60.f;
constexpr int kFzStages = 6;
constexpr int kFzSlots = 16;  // row slots, > 2 * kFzStages - 2
constexpr int kFzMaxRows = 2048;  // rows per chunk (their previous f sits in shared memory)

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

// Shared-memory layout of k_fused_iter after the ring.
struct FusedShared {
    uint64_t full[kFzStages];        // stage landed (producer's transaction count)
    uint64_t empty[kFzStages];       // stage free: 8 row + 8 column warps
    uint64_t wpair_bar[kFzSlots];    // the row's 256 lane pairs posted (8 warp arrivals)
    uint64_t hpair_bar[kFzSlots];    // both halves' pairs present: local arrive + 8 remote bytes
    uint64_t f_bar[kFzSlots];        // f of the row posted
    float2 hpair[kFzSlots][2];       // [cluster rank]: half-row pairs
    float fq[kFzSlots];              // effective f (-inf for a masked row)
    // per row in the ring: each row lane's (max of x = (g - c) k2, sum of
    // 2^(x - max)); the max also bounds the column lane's terms of that row
    float2 lpair[kFzStages][kFzGroup];
    float fin[kFzMaxRows];           // the chunk's previous f, read before any CTA writes f
};

// (max, sum) pairs in log2 units: sum of 2^(x - max).
__device__ __forceinline__ void lse_merge2(float& m, float& s, float m2, float s2) {
    const float mn = fmaxf(m, m2);
    if (mn == -INFINITY) return;
    s = s * ex2(m - mn) + s2 * ex2(m2 - mn);
    m = mn;
}

// softmin = -eps * LSE in natural units, from a log2-unit pair (the guard of
// the reference: an infinite softmin becomes 0, an empty row gives 0).
__device__ __forceinline__ float softmin_from_pair2(float m, float s, float eps) {
    if (m == -INFINITY) return 0.f;
    float sm = -eps * (kLn2 * (m + log2f(s)));
    if (isinf(sm)) sm = 0.f;
    return sm;
}

// natural-unit LSE of a column state (reference cm, sum cs in log2 units)
__device__ __forceinline__ float lse_nat(float cm, float cs) {
    return cs > 0.f ? kLn2 * (cm + log2f(cs)) : -INFINITY;
}

// Row lane t of a staged half-row: float4 groups t + 256 u, x = (g - c) k2.
template <int G4, typename T>
__device__ __forceinline__ float row_lane_max(const T* row, int t, const float (&gk)[4 * G4],
                                              const bool (&gv)[G4], float k2) {
    float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
    for (int u = 0; u < G4; ++u) {
        if (!gv[u]) continue;
        const float4 c = lds_c4<T>(row + (t + kFzGroup * u) * 4);
        m0 = fmaxf(m0, fmaxf((gk[4 * u + 0] - c.x) * k2, (gk[4 * u + 1] - c.y) * k2));
        m1 = fmaxf(m1, fmaxf((gk[4 * u + 2] - c.z) * k2, (gk[4 * u + 3] - c.w) * k2));
    }
    return fmaxf(m0, m1);
}

// One pass: the lane's max of x and the sum of 2^(x - ref). Pairs of columns
// go through the packed fp32x2 pipe: g - c as fma(c, -1, g), then * k2 and
// - ref, each rounded exactly as the scalar operations, so the result is
// bit-identical to the scalar form with half the FP instructions.
template <int G4, typename T>
__device__ __forceinline__ void row_lane_pass(const T* row, int t, const float (&gk)[4 * G4],
                                              const bool (&gv)[G4], float k2, float ref,
                                              float& lm, float& ls) {
    float m0 = -INFINITY, m1 = -INFINITY;
    float2 s01 = make_float2(0.f, 0.f), s23 = make_float2(0.f, 0.f);
    const float2 kk = make_float2(k2, k2), nref = make_float2(-ref, -ref);
    const float2 neg1 = make_float2(-1.f, -1.f);
#pragma unroll
    for (int u = 0; u < G4; ++u) {
        if (!gv[u]) continue;
        const float4 c = lds_c4<T>(row + (t + kFzGroup * u) * 4);
        const float2 x01 = __fmul2_rn(
            __ffma2_rn(make_float2(c.x, c.y), neg1, make_float2(gk[4 * u + 0], gk[4 * u + 1])),
            kk);
        const float2 x23 = __fmul2_rn(
            __ffma2_rn(make_float2(c.z, c.w), neg1, make_float2(gk[4 * u + 2], gk[4 * u + 3])),
            kk);
        m0 = fmaxf(m0, fmaxf(x01.x, x01.y));
        m1 = fmaxf(m1, fmaxf(x23.x, x23.y));
        const float2 d01 = __fadd2_rn(x01, nref), d23 = __fadd2_rn(x23, nref);
        s01 = __fadd2_rn(s01, make_float2(ex2(d01.x), ex2(d01.y)));
        s23 = __fadd2_rn(s23, make_float2(ex2(d23.x), ex2(d23.y)));
    }
    lm = fmaxf(m0, m1);
    ls = (s01.x + s01.y) + (s23.x + s23.y);
}

// G4 = float4 column groups per thread within the CTA's half-row; FULL: the
// half-row is exactly kFzGroup * 4 * G4 columns (no bounds guards).
// 19 warps: one SM sub-partition holds 5 of them, so 16,384 / (5 x 32) caps
// a thread at 96 registers (one CTA per SM).
// T: element type of C (float, or uint16_t holding bf16); the ring holds T.
template <int G4, bool FULL, typename T = float>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kFzThreads, 1)
    k_fused_iter(FusedArgs a) {
    pdl_wait();
    pdl_trigger();
    constexpr int NV = 4 * G4;  // columns per thread
    extern __shared__ __align__(128) unsigned char smem[];
    const int64_t half = a.M >> 1;
    T* ring = reinterpret_cast<T*>(smem);
    FusedShared& S = *reinterpret_cast<FusedShared*>(smem + (size_t)kFzStages * half * sizeof(T));
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
    const int64_t R = r1 > r0 ? r1 - r0 : 0;  // <= kFzMaxRows: the row loops count in 32 bits
    const int64_t col0 = (int64_t)rank * half;
    if (R > kFzMaxRows) {  // the plan never does this; same answer in both CTAs
        if (threadIdx.x == 0 && rank == 0) atomicMax(&st->err, 3);
        return;
    }
    // f is updated in place and both CTAs of a row need its previous value:
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
        mbar_init_fence();
    }
    __syncthreads();
    __syncwarp();
    cluster_barrier();  // the peer's barriers exist before any remote arrive

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp == kFzProducer) {
        // ---- producer: one bulk copy of the half-row per stage -----------
        if (lane == 0 && R > 0) {
            const T* src = reinterpret_cast<const T*>(a.C) + b * a.sCb + r0 * a.sCn + col0;
            int64_t issued = 0;
            for (uint32_t i = 0; i < (uint32_t)R; ++i) {
                const int q = (int)(i % kFzStages);
                if (i >= kFzStages &&
                    !wait_full(&S.empty[q], (uint32_t)((i / kFzStages) - 1) & 1u, &sh_abort)) {
                    sh_abort = 1;
                    break;
                }
                mbar_expect_tx(&S.full[q], (uint32_t)(half * sizeof(T)));
                bulk_g2s(ring + (size_t)q * half, src + i * a.sCn, (uint32_t)(half * sizeof(T)),
                         &S.full[q]);
                issued = i + 1;
            }
            const int64_t first = issued > kFzStages ? issued - kFzStages : 0;
            for (int64_t i = first; i < issued; ++i)
                if (!mbar_wait(&S.full[i % kFzStages], (uint32_t)(i / kFzStages) & 1u))
                    sh_abort = 1;
        }
        __syncwarp();
    } else if (warp < kFzRowWarps) {
        // ---- row warp: (max, sum exp) of its slice of each half-row -------
        const int t = threadIdx.x;
        const float k2 = a.k2;
        float gk[NV];
        bool gv[G4];
#pragma unroll
        for (int u = 0; u < G4; ++u) {
            const int64_t c4 = (int64_t)(t + kFzGroup * u) * 4;  // column in the half
            gv[u] = FULL || c4 < half;
            float4 g4 = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
            if (gv[u]) g4 = ld_vec4(a.g_eff + b * a.M + col0 + c4);
            gk[4 * u + 0] = g4.x;
            gk[4 * u + 1] = g4.y;
            gk[4 * u + 2] = g4.z;
            gk[4 * u + 3] = g4.w;
        }
        float ref = -INFINITY;  // the previous row's lane max (log2 units)
        for (uint32_t i = 0; i < (uint32_t)R; ++i) {
            const int q = (int)(i % kFzStages);
            if (!warp_wait(&S.full[q], (uint32_t)(i / kFzStages) & 1u, &sh_abort)) {
                sh_abort = 1;
                break;
            }
            const T* row = ring + (size_t)q * half;
            if (ref == -INFINITY) ref = row_lane_max<G4>(row, t, gk, gv, k2);  // first row
            float lm, ls;
            row_lane_pass<G4>(row, t, gk, gv, k2, ref == -INFINITY ? 0.f : ref, lm, ls);
            if (lm != -INFINITY && !(lm <= ref + kRefAbove && lm >= ref - kRefBelow)) {
                // rare: the row's max moved far from the reference; sum again
                // against the max itself (the row is still in shared memory)
                ref = lm;
                row_lane_pass<G4>(row, t, gk, gv, k2, ref, lm, ls);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.empty[q]);  // this warp is done with the stage
            // max-normalised pair; an empty lane (lm = -inf) keeps its sum,
            // 0 or NaN, so a NaN cost still reaches f
            const float pair_s = lm == -INFINITY ? ls : ls * ex2((ref == -INFINITY ? 0.f : ref) - lm);
            S.lpair[q][t] = make_float2(lm, pair_s);
            if (lm != -INFINITY) ref = lm;
            __syncwarp();  // every lane's pair store precedes the arrive
            if (lane == 0) mbar_arrive(&S.wpair_bar[(int)(i % kFzSlots)]);
        }
    } else if (warp == kFzSender) {
        // ---- sender: half-row pair, to this CTA and to the peer ----------
        const uint32_t remote_pair0 = map_to_rank(&S.hpair[0][0], peer);
        const uint32_t remote_bar0 = map_to_rank(&S.hpair_bar[0], peer);
        for (uint32_t i = 0; i < (uint32_t)R; ++i) {
            const int sl = (int)(i % kFzSlots);
            if (!warp_wait(&S.wpair_bar[sl], (uint32_t)(i / kFzSlots) & 1u, &sh_abort)) {
                sh_abort = 1;
                break;
            }
            // 256 lane pairs: their max, then the rescaled sum
            const int q = (int)(i % kFzStages);
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
                st_async_f32x2(remote_pair0 + (uint32_t)(sl * 2 + (int)rank) * sizeof(float2), m,
                               sum, remote_bar0 + (uint32_t)sl * sizeof(uint64_t));
                // this CTA's arrival; the phase also waits for the peer's 8 bytes
                mbar_expect_tx(&S.hpair_bar[sl], (uint32_t)sizeof(float2));
            }
            __syncwarp();
        }
    } else if (warp == kFzFinisher) {
        // ---- finisher: f_i from both halves' pairs ------------------------
        float res = 0.f;
        float lav = 0.f;  // this row's scalars, loaded one row ahead
        bool valid = true;
        if (lane == 0 && R > 0) {
            const int64_t g0 = b * a.N + r0;
            lav = __ldg(a.log_a + g0);
            valid = (a.mask_a == nullptr) || (a.mask_a[g0] != 0);
        }
        for (uint32_t i = 0; i < (uint32_t)R; ++i) {
            const int sl = (int)(i % kFzSlots);
            if (!warp_wait_peer(&S.hpair_bar[sl], (uint32_t)(i / kFzSlots) & 1u, &sh_abort)) {
                sh_abort = 1;
                break;
            }
            if (lane == 0) {
                const float fin = S.fin[i];
                const float2 p0 = S.hpair[sl][0];
                const float2 p1 = S.hpair[sl][1];
                float mm = p0.x, ss = p0.y;
                lse_merge2(mm, ss, p1.x, p1.y);  // rank order: identical in both CTAs
                float fo = 0.f;  // masked_fill(~mask_a, 0)
                if (valid) {
                    const float sm = softmin_from_pair2(mm, ss, a.eps);
                    const float fullv = sm + a.eps * lav;
                    fo = (a.rho == 0.f) ? fullv : a.rho * fin + a.omr * fullv;
                }
                const float fe = valid ? fo : -INFINITY;
                S.fq[sl] = fe;
                mbar_arrive(&S.f_bar[sl]);
                if (rank == 0) {
                    const int64_t grow = b * a.N + r0 + i;
                    a.f_out[grow] = fo;
                    a.f_eff[grow] = fe;
                    const float d = fabsf(fo - fin);
                    res = (d > res || isnan(d)) ? d : res;
                }
                if (i + 1 < R) {
                    const int64_t gn = b * a.N + r0 + i + 1;
                    lav = __ldg(a.log_a + gn);
                    valid = (a.mask_a == nullptr) || (a.mask_a[gn] != 0);
                }
            }
            __syncwarp();
        }
        if (lane == 0 && rank == 0) {
            if (b == 0) a.parts[chunk * (a.B * a.M + 4) + a.B * a.M] = 0.f;
            if (check) atomic_max_nonneg(&st->res_bits, res);
        }
        __syncwarp();
    } else if (warp < kFzRowWarps + kFzColWarps) {
        // ---- column warp: fold row i with f_i into the column states -----
        // column lane tc holds float4 groups tc + 256 u of the half-row, the
        // columns of row lane tc (whose max bounds their terms)
        constexpr int CG4 = G4;
        constexpr int CNV = 4 * CG4;
        const int tc = threadIdx.x - kFzGroup;
        const int tr = tc & (kFzGroup - 1);
        const float k2 = a.k2;
        float cm[CNV], cs[CNV];  // per column: reference (log2 units) and sum of 2^(y - cm)
        bool gv[CG4];
#pragma unroll
        for (int u = 0; u < CG4; ++u)
            gv[u] = FULL || (int64_t)(tc + kFzColLanes * u) * 4 < half;
#pragma unroll
        for (int v = 0; v < CNV; ++v) {
            cm[v] = -3.0e38f;  // finite start: an empty column keeps cs = 0
            cs[v] = 0.f;
        }
        // hmin = min over this lane's unmasked columns of g * k2 + cm. Term
        // (f - c) k2 - cm = x + (f - g) k2 - cm <= lmax + f k2 - hmin, with x =
        // (g - c) k2 and lmax row lane tr's max of x over the same columns.
        float hmin = -INFINITY;  // no bound before the first row sets cm
        const float* gsrc = a.g_eff + b * a.M + col0;
        for (uint32_t i = 0; i < (uint32_t)R; ++i) {
            const int sl = (int)(i % kFzSlots);
            if (!warp_wait(&S.f_bar[sl], (uint32_t)(i / kFzSlots) & 1u, &sh_abort)) {
                sh_abort = 1;
                break;
            }
            const float f = S.fq[sl];
            const int q = (int)(i % kFzStages);
            const float bound = S.lpair[q][tr].x + f * k2 - hmin;
            if (!warp_wait(&S.full[q], (uint32_t)(i / kFzStages) & 1u, &sh_abort)) {
                sh_abort = 1;
                break;
            }
            const T* row = ring + (size_t)q * half;
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
                        const float4 c =
                            lds_c4<T>(row + (tc + kFzColLanes * u) * 4);
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const int v = 4 * u + 2 * h;
                            const float2 cc = h ? make_float2(c.z, c.w) : make_float2(c.x, c.y);
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
                        const float4 c =
                            lds_c4<T>(row + (tc + kFzColLanes * u) * 4);
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
                        const float4 g4 = ld_vec4(gsrc + (tc + kFzColLanes * u) * 4);
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
    __syncthreads();
    if (threadIdx.x == 0 && sh_abort) {
        atomicMax(&st->err, 2);
        // a peer waiting for this CTA's pairs stops at once instead of timing out
        st_cluster_u32(map_to_rank((const void*)&sh_abort, peer), 1u);
    }
    __syncwarp();
    cluster_barrier();  // no CTA leaves while its peer may still touch its shared memory
}

// Opt in to more than 48 KB of dynamic shared memory, once per device.
template <int G4, bool FULL, typename T = float>
static int ensure_fused_smem() {
    static thread_local unsigned long long ready = 0;  // bit per device ordinal
    int dev = 0;
    SK_CUDA(cudaGetDevice(&dev));
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(ready & bit)) {
        SK_CUDA(cudaFuncSetAttribute(k_fused_iter<G4, FULL, T>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)(kFzStages * 8192 * sizeof(T) + sizeof(FusedShared))));
        SK_CUDA(cudaFuncSetAttribute(k_fused_iter<G4, FULL, T>,
                                     cudaFuncAttributePreferredSharedMemoryCarveout,
                                     (int)cudaSharedmemCarveoutMaxShared));
        ready |= bit;
    }
    return SK_OK;
}

template <int G4, typename T = float>
static int launch_fused_g(const FusedArgs& a, int64_t nunits, cudaStream_t s) {
    const size_t smem = (size_t)kFzStages * (a.M / 2) * sizeof(T) + sizeof(FusedShared);
    if (a.M / 2 == (int64_t)kFzGroup * 4 * G4) {
        if (int e = ensure_fused_smem<G4, true, T>()) return e;
        launch_pdl(k_fused_iter<G4, true, T>, dim3((unsigned)(2 * nunits)), dim3(kFzThreads),
                   smem, s, a);
        SK_LAUNCHED("k_fused_iter launch");
        return SK_OK;
    }
    if (int e = ensure_fused_smem<G4, false, T>()) return e;
    launch_pdl(k_fused_iter<G4, false, T>, dim3((unsigned)(2 * nunits)), dim3(kFzThreads), smem,
               s, a);
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
    const int smem = (int)(kFzStages * 8192 * 4 + sizeof(FusedShared));
    if (ensure_fused_smem<8, true>() == SK_OK) {
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
        if (cudaOccupancyMaxActiveClusters(&n, k_fused_iter<8, true>, &cfg) != cudaSuccess) n = 0;
    }
    cudaGetLastError();
    if (n <= 0) n = 74;
    cache[dev] = n;
    return n;
}

static bool fused_shape(int64_t N, int64_t M) {
    return M % 8 == 0 && M >= 2048 && M <= 16384 && N >= 1;
}

static int64_t fused_min_chunks(int64_t N) { return (N + kFzMaxRows - 1) / kFzMaxRows; }

int64_t fused_max_chunks(int64_t B, int64_t N, int64_t M) {
    if (rows_fused_shape(N, M)) return rows_fused_max_chunks(B, N);
    if (!fused_shape(N, M)) return 0;
    const int64_t waves = B >= 296 ? 1 : (296 + B - 1) / B;
    return std::max(waves, fused_min_chunks(N));
}

void plan_fused(SweepPlan& p, int64_t B, int64_t N, int64_t M) {
    p.fused = 0;
    p.fused_ok = 0;
    p.fused_rows = 0;
    if (rows_fused_shape(N, M)) {
        // whole rows per CTA (k_rows_fused)
        const int64_t c = rows_fused_chunks(B, N);
        p.rows_per_chunk = (N + c - 1) / c;
        p.chunks = (N + p.rows_per_chunk - 1) / p.rows_per_chunk;
        p.fused_ok = 1;
        p.fused_rows = 1;
        // sk_forward takes it where every SM gets rows to pipeline (measured
        // per iteration against the two sweeps: B=16 N=M=2048 0.078 vs 0.118
        // ms; B=64 N=M=1024 with prefix masks 0.101 vs 0.123 ms); a small batch
        // keeps the sweeps, which spread rows and columns over all SMs
        p.fused = B * N >= 148 * 32 ? 1 : 0;
        return;
    }
    if (!fused_shape(N, M)) return;
    const int64_t A = fused_active_clusters();
    const int64_t cmin = fused_min_chunks(N);
    const int64_t cmax = fused_max_chunks(B, N, M);
    int64_t best_c = cmin;
    double best_eff = -1.0;
    for (int64_t c = cmin; c <= cmax; ++c) {
        if (c > cmin && N / c < 16) break;  // keep chunks at least 16 rows deep
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
    // sk_forward takes the fused iteration where it measured faster on B200
    // (per iteration, fused vs row + column sweep): N=M=16384 0.203 vs 0.383
    // ms, 8192 0.094 vs 0.125, N=4096 M=16384 0.080 vs 0.120. Below M = 8192
    // a thread folds 8 or fewer columns of a row and the per-row exchange
    // dominates (N=65536 M=4096: 0.464 vs 0.395), so those shapes keep the two
    // sweeps; their fused iteration stays available through
    // sk_solver_fused_step / _finish. (M <= 2048 takes k_rows_fused above.)
    p.fused = M >= 8192 ? 1 : 0;
}

int launch_fused(const Problem& P, const SweepPlan& p, const SolveWs& w, const Scalars& sc,
                 const uint8_t* mask_a, float* f, cudaStream_t s) {
    if (p.fused_rows) return launch_rows_fused(P, p, w, sc, mask_a, f, s);
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
    a.k2 = (float)(1.4426950408889634074 / (double)sc.eps);
    a.eps = sc.eps;
    a.rho = sc.rho_a;
    a.omr = sc.omr_a;
    a.st = (Status*)w.status;
    const int64_t nunits = P.B * p.chunks;
    const int64_t g4 = (P.M / 8 + kFzGroup - 1) / kFzGroup;  // float4 groups per thread
    if (p.bf16) {
        if (g4 <= 1) return launch_fused_g<1, uint16_t>(a, nunits, s);
        if (g4 <= 2) return launch_fused_g<2, uint16_t>(a, nunits, s);
        if (g4 <= 4) return launch_fused_g<4, uint16_t>(a, nunits, s);
        return launch_fused_g<8, uint16_t>(a, nunits, s);
    }
    if (g4 <= 1) return launch_fused_g<1>(a, nunits, s);
    if (g4 <= 2) return launch_fused_g<2>(a, nunits, s);
    if (g4 <= 4) return launch_fused_g<4>(a, nunits, s);
    return launch_fused_g<8>(a, nunits, s);
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
