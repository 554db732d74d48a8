// sk_implicit.cu -- the implicit-differentiation adjoint without a stored plan (C ABI).
//
// implicit_gradient (src/sinkhorn/pytorch/implicit_diff.py:196-249) solves
//     (I - J_T^T + reg I) lambda = (grad_f, grad_g)
// by batched conjugate gradients (cg_solve, :107-193) with the Schur matvec of
// :45-104, whose only contact with the plan is P (v_g / c) and P^T (v_f / r),
// r and c being the plan's row and column sums clamped at 1e-30. Here:
//   * k_plan_mv makes one pass over C per product, P recomputed tile by tile
//     from C, f, g (or read from a dense plan when the caller has one), giving
//     P x and P^T y together as partial sums: per (row, column chunk) and per
//     (row band, column). Its exp is exp_scaled (a few ulp): the CG amplifies
//     rounding of the plan by ~1e3, so the cheaper ex2 of a rounded argument
//     is not used here.
//   * a CG iteration is that pass and three element-parallel kernels over the
//     B x (N + M) vectors: k_cg_a merges the partials into A p and p.Ap,
//     k_cg_b updates x and r and r.r, k_cg_c updates p and the next pass's
//     weights xs = p_g / c, ys = p_f / r. The batch dots are double atomics
//     into three rotating slots; the last CTA of k_cg_b takes the stopping
//     decision (max_b |r_b| < tol * max_b |rhs_b|; a NaN never passes) into a
//     device flag that every later launch reads first, so the host queues
//     max_iters iterations with no synchronisation in between.
// Vectors and step scalars are fp32 as in the reference; dots are double.
#include <algorithm>
#include <cmath>

#include "sk_band.cuh"
#include "sk_internal.h"
#include "sk_tma.cuh"

namespace sk {

constexpr float kSumFloor = 1e-30f;   // row_sum / col_sum clamp, implicit_diff.py:83-84
constexpr double kDotFloor = 1e-30;   // pAp and r.r clamps, implicit_diff.py:168,187
constexpr float kMaskedV = -1e20f;    // column potential of masked / absent columns

// ---------------------------------------------------------------------------
// The plan pass: P x and P^T y as partial sums.

constexpr int kMvWarps = 8;                    // consumer warps
constexpr int kMvThreads = 32 * (kMvWarps + 1);  // + one producer warp
constexpr int kMvU = 2;                        // float4 per lane per row
constexpr int kMvW = 128 * kMvU;               // columns per chunk (1 KB of a row)
constexpr int kMvRows = 4;                     // rows per consumer warp per stage
constexpr int kMvStageRows = kMvWarps * kMvRows;  // 32 rows per stage
constexpr int kMvStages = 3;                   // ring depth
constexpr int kMvMinBlocks = 2;                // CTAs per SM (shared memory bound)

struct MvArgs {
    const float* C;        // P-free: the cost (B,N,M), column stride 1
    int64_t sCb, sCn;
    const float* P;        // dense plan (B,N,M) contiguous, or nullptr
    int64_t B, N, M;
    const float* u;        // (B,N) f
    const float* v;        // (B,M) g
    const uint8_t* mask_a; // P-free only
    const uint8_t* mask_b;
    const float* x;        // (B,M) row-sum weights, nullptr = 1
    const float* y;        // (B,N) column-sum weights, nullptr = 1
    float khi, klo;        // log2(e)/eps as a float pair
    float* row_part;       // (B*N, nchunks)
    float* col_part;       // (B, nbands, M)
    float* row_part1;      // DUAL: unweighted row sums, same layout
    float* col_part1;      // DUAL: unweighted column sums
    int64_t nchunks, nbands, band_rows;
    const int* skip;       // device flag: return at once when nonzero
    int* err;              // set to 1 when a wait gives up (never in a healthy run)
};

struct MvSmem {
    float4 ring[kMvStages][kMvStageRows][kMvW / 4];  // 32 KB per stage
    float4 red[kMvWarps][kMvW / 4];                 // column partials of the warps
    float2 rowv[kMvStages][kMvStageRows];           // per row: (f, y), written by the producer
    float4 colv[kMvStages][2][kMvW / 4];            // with a unit's first stage: [0] g (masked: -1e20), [1] x
    unsigned live[kMvStages];                       // bit r: row r of the stage was copied
    uint64_t full[kMvStages];
    uint64_t empty[kMvStages];
    int err;
};

// Sum over the warp of four values per lane, one per row: afterwards lanes
// with (lane & 7) == 0 hold the sums, lane 8 r of row r. A butterfly that
// halves the values carried at each of the first two stages: 6 shuffles for
// four rows instead of 20.
__device__ __forceinline__ float warp_sum4(const float (&v)[4], int lane) {
    const bool hi = lane & 16;
    const float k0 = hi ? v[2] : v[0], k1 = hi ? v[3] : v[1];
    const float s0 = hi ? v[0] : v[2], s1 = hi ? v[1] : v[3];
    const float a0 = k0 + __shfl_xor_sync(0xffffffffu, s0, 16);
    const float a1 = k1 + __shfl_xor_sync(0xffffffffu, s1, 16);
    const bool h8 = lane & 8;
    float r = (h8 ? a1 : a0) + __shfl_xor_sync(0xffffffffu, h8 ? a0 : a1, 8);
    r += __shfl_xor_sync(0xffffffffu, r, 4);
    r += __shfl_xor_sync(0xffffffffu, r, 2);
    r += __shfl_xor_sync(0xffffffffu, r, 1);
    return r;
}

__device__ __forceinline__ bool mv_row_live(const MvArgs& a, bool dense, int64_t b, int64_t i,
                                            int64_t r_hi) {
    if (i >= r_hi) return false;
    return dense || a.mask_a == nullptr || a.mask_a[b * a.N + i] != 0;
}

// One stage of the persistent walk: rows [s0, s0 + 32) of a unit's band.
struct MvStage {
    int64_t unit;   // == units past the end
    int64_t b, j0, s0, r_lo, r_hi;
    uint32_t bytes; // row segment bytes of the unit's chunk
};

__device__ __forceinline__ MvStage mv_first_stage(const MvArgs& a, int64_t unit,
                                                  int64_t units) {
    MvStage st{};
    st.unit = unit;
    if (unit >= units) return st;
    const int64_t chunk = unit % a.nchunks;
    const int64_t t2 = unit / a.nchunks;
    const int64_t band = t2 % a.nbands;
    st.b = t2 / a.nbands;
    st.j0 = chunk * kMvW;
    st.bytes = (uint32_t)(sizeof(float) * (a.M - st.j0 < kMvW ? a.M - st.j0 : kMvW));
    st.s0 = st.r_lo = band * a.band_rows;
    st.r_hi = st.s0 + a.band_rows < a.N ? st.s0 + a.band_rows : a.N;
    return st;
}

__device__ __forceinline__ MvStage mv_next_stage(const MvArgs& a, MvStage st, int64_t units) {
    st.s0 += kMvStageRows;
    if (st.s0 < st.r_hi) return st;
    return mv_first_stage(a, st.unit + gridDim.x, units);
}

// Lane `lane`'s columns of a unit's chunk (j0 + q*128 + lane*4 + {0..3}):
// g with masked / absent columns at -1e20 (P-free), and x (1 when absent).
template <bool DENSE>
__device__ __forceinline__ void mv_col_data(const MvArgs& a, const MvStage& st, int lane,
                                            float4 (&cv)[2][kMvU]) {
#pragma unroll
    for (int q = 0; q < kMvU; ++q) {
        const int64_t j = st.j0 + q * 128 + lane * 4;
        const bool in = j < a.M;  // M % 4 == 0: whole float4 in or out
        float4 vv = make_float4(0.f, 0.f, 0.f, 0.f), xx = make_float4(1.f, 1.f, 1.f, 1.f);
        if (in && !DENSE) vv = *reinterpret_cast<const float4*>(a.v + st.b * a.M + j);
        if (in && a.x) xx = *reinterpret_cast<const float4*>(a.x + st.b * a.M + j);
        if (!DENSE) {
            const uint8_t* mb = a.mask_b ? a.mask_b + st.b * a.M + j : nullptr;
            if (!in || (mb && mb[0] == 0)) vv.x = kMaskedV;
            if (!in || (mb && mb[1] == 0)) vv.y = kMaskedV;
            if (!in || (mb && mb[2] == 0)) vv.z = kMaskedV;
            if (!in || (mb && mb[3] == 0)) vv.w = kMaskedV;
        }
        cv[0][q] = vv;
        cv[1][q] = xx;
    }
}

// Row `lane` of a stage: copied or not, and its (f, y) for the consumers.
template <bool DENSE>
__device__ __forceinline__ void mv_row_data(const MvArgs& a, const MvStage& st, int lane,
                                            bool* live, float2* rv) {
    const int64_t i = st.s0 + lane;
    *live = mv_row_live(a, DENSE, st.b, i, st.r_hi);
    *rv = make_float2(kMaskedV, 0.f);
    if (*live) {
        rv->x = DENSE ? 0.f : a.u[st.b * a.N + i];
        rv->y = a.y ? a.y[st.b * a.N + i] : 1.f;
    }
}

__device__ __forceinline__ void consumers_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(32 * kMvWarps) : "memory");
}

// Persistent CTAs loop over units (batch item, row band, column chunk of kMvW
// columns); all roles walk the same unit and stage sequence.
//   * producer warp: per stage of 32 rows, one cp.async.bulk of the chunk's
//     row segment per live row (lane r copies row r), completing on the
//     stage's full mbarrier; masked rows and rows past the band are not read.
//   * 8 consumer warps: 4 rows of the stage each, 8 columns per lane (two
//     float4 from shared memory), the chunk's g, x and column accumulators in
//     registers; row sums by one 4-row butterfly, written per (row, chunk);
//     then an arrive on the stage's empty mbarrier. Column sums: reduced over
//     the warps in shared memory at the end of the unit, one partial per
//     (band, column).
// Masked columns and columns past M get the potential -1e20 and rows not
// copied read as 0 with the potential -1e20, so every such exp is exactly 0
// with no select (a NaN cost at a masked column still gives NaN, as in the
// forward kernels). Every wait is bounded: on a timeout the CTA records the
// error, stops waiting, lets its own copies land and returns.
// TIMES_C: the terms are p * C (the cost <P, C>, sinkhorn.py:56-67).
template <bool DENSE, bool DUAL = false, bool TIMES_C = false>
__global__ void __launch_bounds__(kMvThreads, kMvMinBlocks) k_plan_mv(MvArgs a) {
    if (a.skip != nullptr && *a.skip != 0) return;  // set by an earlier launch on the stream
    extern __shared__ __align__(128) unsigned char mv_smem_raw[];
    MvSmem& S = *reinterpret_cast<MvSmem*>(mv_smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int q = 0; q < kMvStages; ++q) {
            mbar_init(&S.full[q], 1);
            mbar_init(&S.empty[q], kMvWarps);
        }
        S.err = 0;
        mbar_init_fence();
    }
    __syncthreads();

    const int64_t units = a.B * a.nbands * a.nchunks;
    if (warp == kMvWarps) {
        // ---- producer ----------------------------------------------------
        // Walks the stages in order with the next stage's row data (mask,
        // f, y) loaded one stage ahead, so no stage waits on those loads.
        MvStage cur = mv_first_stage(a, blockIdx.x, units);
        bool live_cur = false;
        float2 rv_cur = make_float2(kMaskedV, 0.f);
        float4 cv_cur[2][kMvU];
        if (cur.unit < units) {
            mv_row_data<DENSE>(a, cur, lane, &live_cur, &rv_cur);
            mv_col_data<DENSE>(a, cur, lane, cv_cur);
        }
        uint32_t g = 0;  // stages issued
        bool ok = true;
        for (; cur.unit < units; ++g) {
            const int q = (int)(g % kMvStages);
            if (g >= (uint32_t)kMvStages) {
                ok = mbar_wait(&S.empty[q], ((g / kMvStages) - 1) & 1u);
                if (!ok) break;
            }
            const unsigned bits = __ballot_sync(0xffffffffu, live_cur);
            if (lane == 0) mbar_expect_tx_only(&S.full[q], __popc(bits) * cur.bytes);
            __syncwarp();
            if (live_cur) {
                const int64_t i = cur.s0 + lane;
                const float* src = DENSE ? a.P + (cur.b * a.N + i) * a.M + cur.j0
                                         : a.C + cur.b * a.sCb + i * a.sCn + cur.j0;
                bulk_g2s(&S.ring[q][lane][0], src, cur.bytes, &S.full[q]);
            }
            const MvStage nxt = mv_next_stage(a, cur, units);
            bool live_nxt = false;
            float2 rv_nxt = make_float2(kMaskedV, 0.f);
            float4 cv_nxt[2][kMvU];
            const bool new_unit = nxt.unit < units && nxt.s0 == nxt.r_lo;
            if (nxt.unit < units) mv_row_data<DENSE>(a, nxt, lane, &live_nxt, &rv_nxt);
            if (new_unit) mv_col_data<DENSE>(a, nxt, lane, cv_nxt);
            // the row constants (and a unit's column constants, with its
            // first stage) travel in the stage's slot: plain shared stores
            // ordered before the arrive (release), seen by the consumers after
            // their wait (acquire), rewritten only after the slot's release
            S.rowv[q][lane] = rv_cur;
            if (cur.s0 == cur.r_lo) {
#pragma unroll
                for (int qq = 0; qq < kMvU; ++qq) {
                    S.colv[q][0][qq * 32 + lane] = cv_cur[0][qq];
                    S.colv[q][1][qq * 32 + lane] = cv_cur[1][qq];
                }
            }
            if (lane == 0) S.live[q] = bits;
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.full[q]);
            cur = nxt;
            live_cur = live_nxt;
            rv_cur = rv_nxt;
            if (new_unit) {
#pragma unroll
                for (int qq = 0; qq < kMvU; ++qq) {
                    cv_cur[0][qq] = cv_nxt[0][qq];
                    cv_cur[1][qq] = cv_nxt[1][qq];
                }
            }
        }
        if (!ok) {
            if (lane == 0) {
                S.err = 1;
                atomicExch(a.err, 1);
            }
            // let this CTA's copies land before it exits (bounded)
            const uint32_t lo = g > (uint32_t)kMvStages ? g - kMvStages : 0u;
            for (uint32_t h = lo; h < g; ++h)
                mbar_wait(&S.full[h % kMvStages], (h / kMvStages) & 1u);
        }
        return;
    }

    // ---- consumers -------------------------------------------------------
    uint32_t g = 0;  // stages consumed
    for (int64_t unit = blockIdx.x; unit < units; unit += gridDim.x) {
        const int64_t chunk = unit % a.nchunks;
        const int64_t t2 = unit / a.nchunks;
        const int64_t band = t2 % a.nbands;
        const int64_t b = t2 / a.nbands;

        // per lane: columns j0 + q*128 + lane*4 + {0..3}, as pairs h = {0,1},
        // {2,3}; read from colv once the unit's first stage has arrived
        float2 vj[kMvU][2], xj[kMvU][2], cs[kMvU][2], cs1[kMvU][2];
        bool cin[kMvU];
#pragma unroll
        for (int q = 0; q < kMvU; ++q) {
            cin[q] = chunk * kMvW + q * 128 + lane * 4 < a.M;
            cs[q][0] = cs[q][1] = make_float2(0.f, 0.f);
            cs1[q][0] = cs1[q][1] = make_float2(0.f, 0.f);
        }
        const float2 nkhi = make_float2(-a.khi, -a.khi), nklo = make_float2(-a.klo, -a.klo);
        const float2 khi2 = make_float2(a.khi, a.khi), ln2 = make_float2(kLn2, kLn2);
        const float2 m1 = make_float2(-1.f, -1.f);

        const int64_t r_lo = band * a.band_rows;
        const int64_t r_hi = r_lo + a.band_rows < a.N ? r_lo + a.band_rows : a.N;
        for (int64_t s0 = r_lo; s0 < r_hi; s0 += kMvStageRows, ++g) {
            const int qs = (int)(g % kMvStages);
            if (!*(volatile int*)&S.err && !mbar_wait(&S.full[qs], (g / kMvStages) & 1u)) {
                S.err = 1;
                atomicExch(a.err, 1);
            }
            const bool bad = *(volatile int*)&S.err != 0;
            if (s0 == r_lo) {
#pragma unroll
                for (int q = 0; q < kMvU; ++q) {
                    const float4 vv = S.colv[qs][0][q * 32 + lane];
                    const float4 xx = S.colv[qs][1][q * 32 + lane];
                    vj[q][0] = make_float2(vv.x, vv.y);
                    vj[q][1] = make_float2(vv.z, vv.w);
                    xj[q][0] = make_float2(xx.x, xx.y);
                    xj[q][1] = make_float2(xx.z, xx.w);
                }
            }
            const unsigned bits = bad ? 0u : S.live[qs] >> (warp * kMvRows);
            float rs[kMvRows], rs1[kMvRows];
            float ui[kMvRows], yi[kMvRows];
            bool live[kMvRows];
#pragma unroll
            for (int r = 0; r < kMvRows; ++r) {
                const float2 rv = S.rowv[qs][warp * kMvRows + r];
                live[r] = (bits >> r) & 1u;
                ui[r] = rv.x;
                yi[r] = rv.y;
                rs[r] = rs1[r] = 0.f;
            }
#pragma unroll
            for (int r = 0; r < kMvRows; ++r) {
                if (!live[r]) continue;  // warp-uniform
                const float2 u2 = make_float2(ui[r], ui[r]), y2 = make_float2(yi[r], yi[r]);
                float2 racc = make_float2(0.f, 0.f), racc1 = make_float2(0.f, 0.f);
#pragma unroll
                for (int q = 0; q < kMvU; ++q) {
                    float4 c4 = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (cin[q]) c4 = S.ring[qs][warp * kMvRows + r][q * 32 + lane];
                    const float2 cp[2] = {make_float2(c4.x, c4.y), make_float2(c4.z, c4.w)};
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        float2 p;
                        if constexpr (DENSE) {
                            p = cp[h];
                        } else {
                            // exp_scaled on a pair, in the negated form that
                            // needs no extra negations: nd = C - (f + g) = -d,
                            // ny = -y, t = d khi - y (exact), ylo = t + d klo
                            const float2 nd = __ffma2_rn(__fadd2_rn(u2, vj[q][h]), m1, cp[h]);
                            const float2 ny = __fmul2_rn(nd, khi2);
                            const float2 t = __ffma2_rn(nd, nkhi, ny);
                            float2 corr = __fmul2_rn(__ffma2_rn(nd, nklo, t), ln2);
                            // infinite / NaN arguments: a bounded correction
                            // keeps exp(-inf) = 0, exp(inf) = inf, NaN = NaN
                            corr.x = fmaxf(fminf(corr.x, 0.25f), -0.25f);
                            corr.y = fmaxf(fminf(corr.y, 0.25f), -0.25f);
                            const float2 e = make_float2(ex2(-ny.x), ex2(-ny.y));
                            p = __ffma2_rn(e, corr, e);
                        }
                        if constexpr (TIMES_C) p = __fmul2_rn(p, cp[h]);
                        racc = __ffma2_rn(p, xj[q][h], racc);
                        cs[q][h] = __ffma2_rn(p, y2, cs[q][h]);
                        if constexpr (DUAL) {
                            racc1 = __fadd2_rn(racc1, p);
                            cs1[q][h] = __fadd2_rn(cs1[q][h], p);
                        }
                    }
                }
                rs[r] = racc.x + racc.y;
                if constexpr (DUAL) rs1[r] = racc1.x + racc1.y;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.empty[qs]);  // this warp is done with the stage
            if (a.row_part && !bad) {
                const float rsum = warp_sum4(rs, lane);
                const int64_t i = s0 + warp * kMvRows + (lane >> 3);
                if ((lane & 7) == 0 && i < r_hi)
                    a.row_part[(b * a.N + i) * a.nchunks + chunk] = rsum;
                if constexpr (DUAL) {
                    const float rsum1 = warp_sum4(rs1, lane);
                    if ((lane & 7) == 0 && i < r_hi)
                        a.row_part1[(b * a.N + i) * a.nchunks + chunk] = rsum1;
                }
            }
        }
        if (a.col_part != nullptr) {  // uniform over the consumers
#pragma unroll
            for (int pass = 0; pass < (DUAL ? 2 : 1); ++pass) {
                // the weighted sums, then (DUAL) the plain ones, through S.red
#pragma unroll
                for (int q = 0; q < kMvU; ++q) {
                    const float2 c0 = pass ? cs1[q][0] : cs[q][0];
                    const float2 c1 = pass ? cs1[q][1] : cs[q][1];
                    S.red[warp][q * 32 + lane] = make_float4(c0.x, c0.y, c1.x, c1.y);
                }
                consumers_sync();
                const float* shf = reinterpret_cast<const float*>(S.red);
                float* out = pass ? a.col_part1 : a.col_part;
                for (int cc = threadIdx.x; cc < kMvW; cc += 32 * kMvWarps) {
                    const int64_t j = chunk * kMvW + cc;
                    if (j >= a.M) continue;
                    float sum = 0.f;
#pragma unroll
                    for (int w = 0; w < kMvWarps; ++w) sum += shf[w * kMvW + cc];
                    out[(b * a.nbands + band) * a.M + j] = sum;
                }
                consumers_sync();  // S.red is rewritten next
            }
        }
    }
}

// The plan operator and the layout of one pass's partial sums.
struct PlanOp {
    BandArgs band;      // fallback pass (strided C or M % 4 != 0)
    MvArgs mv;          // k_plan_mv pass
    bool use_mv;
    int64_t nchunks, nbands;
};

// Row bands: enough units for about four per resident CTA (load balance of
// the persistent loop), bands of at least 128 rows (column partials stay a
// small fraction of the pass's traffic), whole warp steps.
static int64_t mv_bands(int64_t B, int64_t N, int64_t nchunks, int64_t* band_rows) {
    const int64_t target = 148 * kMvMinBlocks * 4;
    const int64_t units = B * nchunks;
    const int64_t nb = std::max<int64_t>(1, (target + units - 1) / units);
    constexpr int64_t step = kMvStageRows;
    int64_t br = (N + nb - 1) / nb;
    br = std::max<int64_t>(br, 4 * step);
    br = (br + step - 1) / step * step;
    *band_rows = br;
    return (N + br - 1) / br;
}

static int make_op(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb, int64_t sCn,
                   int64_t sCm, const float* f, const float* g, double epsilon,
                   const uint8_t* mask_a, const uint8_t* mask_b, const float* P, PlanOp* op) {
    *op = PlanOp{};
    if (P) {
        if (int e = check_problem(P, B, N, M, 1.0)) return e;
        op->band = band_base(P, B, N, M, N * M, M, 1, 1.0);
        op->band.P = P;
        op->use_mv = dense_ok(P, M);
    } else {
        if (int e = check_problem(C, B, N, M, epsilon)) return e;
        if (!f || !g) return fail(SK_ERR_ARG, "f and g must be non-NULL without a dense plan");
        op->band = band_base(C, B, N, M, sCb, sCn, sCm, epsilon);
        op->band.precise = 1;
        op->band.u = f;
        op->band.v = g;
        op->band.mask_a = mask_a;
        op->band.mask_b = mask_b;
        op->use_mv = vec4_ok(C, B, M, sCb, sCn, sCm) && ((uintptr_t)g % 16 == 0);
    }
    MvArgs& m = op->mv;
    m.C = C;
    m.sCb = sCb;
    m.sCn = sCn;
    m.P = P;
    m.B = B;
    m.N = N;
    m.M = M;
    m.u = f;
    m.v = g;
    m.mask_a = mask_a;
    m.mask_b = mask_b;
    m.khi = op->band.khi;
    m.klo = op->band.klo;
    if (op->use_mv) {
        op->nchunks = (M + kMvW - 1) / kMvW;
        op->nbands = mv_bands(B, N, op->nchunks, &m.band_rows);
    } else {
        op->nchunks = 1;  // the band pass writes finished sums
        op->nbands = 1;
    }
    m.nchunks = op->nchunks;
    m.nbands = op->nbands;
    return SK_OK;
}

// Dynamic shared memory beyond 48 KB, set once per process for both instances.
static int mv_smem_setup() {
    static int done = 0;
    if (done) return SK_OK;
    SK_CUDA(cudaFuncSetAttribute(k_plan_mv<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)sizeof(MvSmem)));
    SK_CUDA(cudaFuncSetAttribute(k_plan_mv<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)sizeof(MvSmem)));
    SK_CUDA(cudaFuncSetAttribute(k_plan_mv<false, true>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(MvSmem)));
    SK_CUDA(cudaFuncSetAttribute(k_plan_mv<false, false, true>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(MvSmem)));
    SK_CUDA(cudaFuncSetAttribute(k_plan_mv<true>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 (int)cudaSharedmemCarveoutMaxShared));
    SK_CUDA(cudaFuncSetAttribute(k_plan_mv<false>,
                                 cudaFuncAttributePreferredSharedMemoryCarveout,
                                 (int)cudaSharedmemCarveoutMaxShared));
    done = 1;
    return SK_OK;
}

// One pass: P x into row_part and P^T y into col_part (weights nullptr = 1).
// `x` must be 16-byte aligned (k_plan_mv reads it as float4).
static int run_pass(const PlanOp& op, const float* x, const float* y, float* row_part,
                    float* col_part, const int* skip, int* err, void* band_ws, cudaStream_t s) {
    if (op.use_mv) {
        MvArgs m = op.mv;
        m.x = x;
        m.y = y;
        m.row_part = row_part;
        m.col_part = col_part;
        m.skip = skip;
        m.err = err;
        if (int e = mv_smem_setup()) return e;
        const int64_t units = m.B * m.nbands * m.nchunks;
        const unsigned grid = (unsigned)std::min<int64_t>(units, 148 * kMvMinBlocks);
        if (m.P) k_plan_mv<true><<<grid, kMvThreads, sizeof(MvSmem), s>>>(m);
        else k_plan_mv<false><<<grid, kMvThreads, sizeof(MvSmem), s>>>(m);
        SK_LAUNCHED("k_plan_mv launch");
        return SK_OK;
    }
    BandArgs a = op.band;
    a.wc = x;
    a.wr = y;
    a.row_q = row_part ? 2 : 0;
    a.col_q = col_part ? 2 : 0;
    a.row_out0 = row_part;
    a.col_out0 = col_part;
    a.skip = skip;
    return launch_band(a, false, band_ws, s);
}

__device__ __forceinline__ float merge_row(const float* part, int64_t row, int64_t nchunks) {
    float s = 0.f;
    for (int64_t c = 0; c < nchunks; ++c) s += part[row * nchunks + c];
    return s;
}

__device__ __forceinline__ float merge_col(const float* part, int64_t b, int64_t j, int64_t M,
                                           int64_t nbands) {
    float s = 0.f;
    for (int64_t q = 0; q < nbands; ++q) s += part[(b * nbands + q) * M + j];
    return s;
}

// Finished sums of a pass: out_f[b,i] = sum over chunks (nf = B*N entries, 0
// for none), out_g[b,j] = sum over bands (ng = B*M entries, 0 for none).
__global__ void k_mv_merge(const float* row_part, const float* col_part, int64_t nf,
                           int64_t ng, int64_t M, int64_t nchunks, int64_t nbands,
                           float* out_f, float* out_g) {
    const int64_t n = nf + ng;
    for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n;
         k += (int64_t)gridDim.x * blockDim.x) {
        if (k < nf) {
            out_f[k] = merge_row(row_part, k, nchunks);
        } else {
            const int64_t kk = k - nf, b = kk / M, j = kk - b * M;
            out_g[kk] = merge_col(col_part, b, j, M, nbands);
        }
    }
}

static unsigned elem_grid(int64_t n) {
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148 * 8));
}

// ---------------------------------------------------------------------------
// Conjugate gradients (cg_solve, implicit_diff.py:107-193)

constexpr int kCgThreads = 256;
constexpr int kCgPer = 4;                          // elements per thread
constexpr int kCgTile = kCgThreads * kCgPer;       // elements per CTA

struct CgState {
    int done;          // nonzero: converged or out of iterations
    int n_iters;       // iterations taken
    unsigned ticket;   // last-CTA ticket of the current launch
    float rhs_norm;    // max over the batch of |rhs_b|
};
static_assert(sizeof(CgState) == 16, "the dot slots follow the 16-byte state");

struct CgArgs {
    int64_t B, N, M, L;   // L = N + M: one batch item's [f | g] vector
    int64_t pieces;       // CTAs per batch item
    const float* row_part;
    const float* col_part;
    int64_t nchunks, nbands;
    float* rs;            // (B,N) plan row sums
    float* cs;            // (B,M) plan column sums
    const float* rhs_f;
    const float* rhs_g;
    float* x_f;           // solution
    float* x_g;
    float* r_f;           // residual
    float* r_g;
    float* p_f;           // search direction
    float* p_g;
    float* ys;            // (B,N) p_f / r: column-sum weights of the next pass
    float* xs;            // (B,M) p_g / c: row-sum weights of the next pass
    float* ap_f;          // A p
    float* ap_g;
    float* grad_a;        // eps * x_f, or nullptr
    float* grad_b;
    float eps;
    float rho_a, rho_b, reg, tol;
    int max_iters;
    double* acc;          // [3][B][2]: p.Ap and r.r of iteration k in slot k % 3
    int slot;             // k % 3 (k_cg_init: the r.r of the start goes to slot 2)
    CgState* st;
};

__device__ __forceinline__ double clamp_dot(double v) { return v < kDotFloor ? kDotFloor : v; }

// Sum over the CTA; the result is valid in thread 0.
__device__ double cta_sum_d(double v) {
    __shared__ double sh[kCgThreads / 32];
    v = warp_sum_d(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) sh[w] = v;
    __syncthreads();
    double t = 0.0;
    if (w == 0) {
        t = l < kCgThreads / 32 ? sh[l] : 0.0;
        t = warp_sum_d(t);
    }
    __syncthreads();  // sh may be reused
    return t;
}

// True in the last CTA of the launch to arrive (all earlier CTAs' writes,
// atomics included, are visible to it); that CTA resets the ticket.
__device__ bool arrive_last(CgState* st, unsigned ctas) {
    __shared__ int last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(&st->ticket, 1u) == ctas - 1;
    __syncthreads();
    if (last) __threadfence();
    return last != 0;
}

// max_b sqrt(acc[slot][b][1]) over the CTA, NaN-propagating (torch.max).
__device__ float batch_norm_max(const double* acc, int64_t B, int slot) {
    __shared__ float sh[kCgThreads / 32];
    float m = -INFINITY;
    bool nan = false;
    for (int64_t b = threadIdx.x; b < B; b += kCgThreads) {
        const float v = (float)sqrt(__ldcg(acc + ((int64_t)slot * B + b) * 2 + 1));
        nan |= isnan(v);
        m = fmaxf(m, v);
    }
    m = warp_max(m);
    nan = __any_sync(0xffffffffu, nan);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) sh[w] = nan ? NAN : m;
    __syncthreads();
    float r = -INFINITY;
    for (int q = 0; q < kCgThreads / 32; ++q) r = (sh[q] > r || isnan(sh[q])) ? sh[q] : r;
    return r;
}

// Position k of this thread's e-th element in its batch item's [f | g] vector
// (CTA = one batch item, one tile of kCgTile positions), or -1.
__device__ __forceinline__ int64_t cg_pos(const CgArgs& a, int e) {
    const int64_t k = (blockIdx.x % a.pieces) * kCgTile + threadIdx.x + (int64_t)e * kCgThreads;
    return k < a.L ? k : -1;
}

// Start: merge the sums pass into r, c; x = 0, r = p = rhs; the weights of the
// first pass; r.r of the start into slot 2; the last CTA takes max_b |rhs_b|.
__global__ void __launch_bounds__(kCgThreads) k_cg_init(CgArgs a) {
    const int64_t b = blockIdx.x / a.pieces;
    double acc = 0.0;
#pragma unroll
    for (int e = 0; e < kCgPer; ++e) {
        const int64_t k = cg_pos(a, e);
        if (k < 0) continue;
        float v;
        if (k < a.N) {
            const int64_t o = b * a.N + k;
            const float sum = merge_row(a.row_part, o, a.nchunks);
            a.rs[o] = sum;
            v = a.rhs_f[o];
            a.x_f[o] = 0.f;
            a.r_f[o] = v;
            a.p_f[o] = v;
            a.ys[o] = v / fmaxf(sum, kSumFloor);
            if (a.grad_a) a.grad_a[o] = 0.f;
        } else {
            const int64_t j = k - a.N, o = b * a.M + j;
            const float sum = merge_col(a.col_part, b, j, a.M, a.nbands);
            a.cs[o] = sum;
            v = a.rhs_g[o];
            a.x_g[o] = 0.f;
            a.r_g[o] = v;
            a.p_g[o] = v;
            a.xs[o] = v / fmaxf(sum, kSumFloor);
            if (a.grad_b) a.grad_b[o] = 0.f;
        }
        acc += (double)v * v;
    }
    const double t = cta_sum_d(acc);
    if (threadIdx.x == 0) atomicAdd(a.acc + ((int64_t)2 * a.B + b) * 2 + 1, t);
    if (!arrive_last(a.st, gridDim.x)) return;
    const float mx = batch_norm_max(a.acc, a.B, 2);
    if (threadIdx.x == 0) {
        a.st->rhs_norm = mx;
        a.st->n_iters = 0;
        a.st->done = a.max_iters <= 0;
        a.st->ticket = 0u;
    }
}

// A p = (1 + reg) p - J_T^T p from the pass (schur_complement_matvec, :97-102)
// and p.Ap into slot k % 3.
__global__ void __launch_bounds__(kCgThreads) k_cg_a(CgArgs a) {
    if (a.st->done) return;  // written by an earlier launch on the stream
    const int64_t b = blockIdx.x / a.pieces;
    const float ca = 1.f + a.reg;
    double acc = 0.0;
#pragma unroll
    for (int e = 0; e < kCgPer; ++e) {
        const int64_t k = cg_pos(a, e);
        if (k < 0) continue;
        float p, ap;
        if (k < a.N) {
            const int64_t o = b * a.N + k;
            const float q = merge_row(a.row_part, o, a.nchunks);
            p = a.p_f[o];
            ap = ca * p - (a.rho_a * p + (1.f - a.rho_b) * q);
            a.ap_f[o] = ap;
        } else {
            const int64_t j = k - a.N, o = b * a.M + j;
            const float q = merge_col(a.col_part, b, j, a.M, a.nbands);
            p = a.p_g[o];
            ap = ca * p - (a.rho_b * p + (1.f - a.rho_a) * q);
            a.ap_g[o] = ap;
        }
        acc += (double)p * ap;
    }
    const double t = cta_sum_d(acc);
    if (threadIdx.x == 0) atomicAdd(a.acc + ((int64_t)a.slot * a.B + b) * 2, t);
}

// alpha = r.r / max(p.Ap, 1e-30); x += alpha p; r -= alpha A p; r.r into slot
// k % 3. The last CTA: iteration count, stopping test, clears slot (k+1) % 3.
__global__ void __launch_bounds__(kCgThreads) k_cg_b(CgArgs a) {
    if (a.st->done) return;
    const int64_t b = blockIdx.x / a.pieces;
    const int prev = (a.slot + 2) % 3;
    const double rd = __ldcg(a.acc + ((int64_t)prev * a.B + b) * 2 + 1);
    const double pap = __ldcg(a.acc + ((int64_t)a.slot * a.B + b) * 2);
    const float alpha = (float)(rd / clamp_dot(pap));
    double acc = 0.0;
#pragma unroll
    for (int e = 0; e < kCgPer; ++e) {
        const int64_t k = cg_pos(a, e);
        if (k < 0) continue;
        float r;
        if (k < a.N) {
            const int64_t o = b * a.N + k;
            const float x = a.x_f[o] + alpha * a.p_f[o];
            r = a.r_f[o] - alpha * a.ap_f[o];
            a.x_f[o] = x;
            a.r_f[o] = r;
            if (a.grad_a) a.grad_a[o] = a.eps * x;
        } else {
            const int64_t o = b * a.M + (k - a.N);
            const float x = a.x_g[o] + alpha * a.p_g[o];
            r = a.r_g[o] - alpha * a.ap_g[o];
            a.x_g[o] = x;
            a.r_g[o] = r;
            if (a.grad_b) a.grad_b[o] = a.eps * x;
        }
        acc += (double)r * r;
    }
    const double t = cta_sum_d(acc);
    if (threadIdx.x == 0) atomicAdd(a.acc + ((int64_t)a.slot * a.B + b) * 2 + 1, t);
    if (!arrive_last(a.st, gridDim.x)) return;
    const float res = batch_norm_max(a.acc, a.B, a.slot);
    const int next = (a.slot + 1) % 3;
    for (int64_t q = threadIdx.x; q < 2 * a.B; q += kCgThreads)
        a.acc[(int64_t)next * a.B * 2 + q] = 0.0;
    if (threadIdx.x == 0) {
        const int n = a.st->n_iters + 1;
        a.st->n_iters = n;
        if (res < a.tol * a.st->rhs_norm || n >= a.max_iters) a.st->done = 1;
        a.st->ticket = 0u;
    }
}

// beta = r'.r' / max(r.r, 1e-30); p = r + beta p; the next pass's weights.
__global__ void __launch_bounds__(kCgThreads) k_cg_c(CgArgs a) {
    if (a.st->done) return;
    const int64_t b = blockIdx.x / a.pieces;
    const int prev = (a.slot + 2) % 3;
    const double rn = __ldcg(a.acc + ((int64_t)a.slot * a.B + b) * 2 + 1);
    const double rd = __ldcg(a.acc + ((int64_t)prev * a.B + b) * 2 + 1);
    const float beta = (float)(rn / clamp_dot(rd));
#pragma unroll
    for (int e = 0; e < kCgPer; ++e) {
        const int64_t k = cg_pos(a, e);
        if (k < 0) continue;
        if (k < a.N) {
            const int64_t o = b * a.N + k;
            const float p = a.r_f[o] + beta * a.p_f[o];
            a.p_f[o] = p;
            a.ys[o] = p / fmaxf(a.rs[o], kSumFloor);
        } else {
            const int64_t o = b * a.M + (k - a.N);
            const float p = a.r_g[o] + beta * a.p_g[o];
            a.p_g[o] = p;
            a.xs[o] = p / fmaxf(a.cs[o], kSumFloor);
        }
    }
}

// ---------------------------------------------------------------------------
// Single matvecs (sk_implicit_matvec)

enum MatvecMode : int {
    MV_SCHUR = 0,  // (1 + reg) v - J_T^T v               implicit_diff.py:45-104
    MV_VJP = 1,    // J_T^T v, 0 at masked entries          implicit_diff.py:281-309
    MV_JVP = 2,    // J_T v, 0 at masked entries            implicit_diff.py:253-278
};

// Weights of the pass: v_f / r and v_g / c (SCHUR, VJP) or v_f, v_g (JVP).
__global__ void k_mv_weights(const float* v, const float* sums, int64_t n, int scaled,
                             float* out) {
    for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n;
         k += (int64_t)gridDim.x * blockDim.x)
        out[k] = scaled ? v[k] / fmaxf(sums[k], kSumFloor) : v[k];
}

// out = tail(v, q) on one side; rho_s is this side's rho, omr the factor of
// the pass result ((1 - rho_other) for the transpose, (1 - rho_s) for J_T).
__global__ void k_mv_out(const float* v, const float* q, const float* sums,
                         const uint8_t* mask, int64_t n, int mode, float rho_s, float omr,
                         float ca, float* out) {
    for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n;
         k += (int64_t)gridDim.x * blockDim.x) {
        const float vk = v[k];
        float o;
        if (mode == MV_SCHUR) {
            o = ca * vk - (rho_s * vk + omr * q[k]);
        } else if (mode == MV_VJP) {
            o = rho_s * vk + omr * q[k];
        } else {
            o = rho_s * vk + omr * q[k] / fmaxf(sums[k], kSumFloor);
        }
        if (mode != MV_SCHUR && mask != nullptr && mask[k] == 0) o = 0.f;
        out[k] = o;
    }
}

// ---------------------------------------------------------------------------
// dC_ij = -(1/eps) P_ij (lf_i + lg_j), P = exp((f_i + g_j - C_ij)/eps) from
// exp_scaled as in the CG passes, 0 at masked rows / columns
// (implicit_gradient, implicit_diff.py:241-243). A warp per row, grid-stride
// over the B*N rows: one read of C, one streaming write.
template <int VEC>
__global__ void __launch_bounds__(256) k_implicit_dc(
    const float* C, int64_t sCb, int64_t sCn, int64_t sCm, int64_t B, int64_t N, int64_t M,
    const float* f, const float* g, const float* lf, const float* lg, const uint8_t* mask_a,
    const uint8_t* mask_b, float khi, float klo, float inv_eps, float* dC) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
         row < B * N; row += warps) {
        const int64_t b = row / N, i = row - b * N;
        const bool rvalid = mask_a == nullptr || mask_a[row] != 0;
        const float fi = f[row], lfi = lf[row];
        const float* Crow = C + b * sCb + i * sCn;
        const float* gb = g + b * M;
        const float* lgb = lg + b * M;
        const uint8_t* mb = mask_b ? mask_b + b * M : nullptr;
        float* out = dC + row * M;
        for (int64_t j0 = (int64_t)lane * VEC; j0 < M; j0 += 32 * VEC) {
            float c[VEC] = {}, o[VEC];
            if (rvalid) {
                if constexpr (VEC == 4) {
                    const float4 cc = ld_stream4(Crow + j0);
                    c[0] = cc.x; c[1] = cc.y; c[2] = cc.z; c[3] = cc.w;
                } else {
                    c[0] = ld_stream1(Crow + j0 * sCm);
                }
            }
#pragma unroll
            for (int q = 0; q < VEC; ++q) {
                const int64_t j = j0 + q;
                o[q] = 0.f;
                if (rvalid && (mb == nullptr || mb[j] != 0)) {
                    const float p = exp_scaled((fi + gb[j]) - c[q], khi, klo);
                    o[q] = -inv_eps * p * (lfi + lgb[j]);
                }
            }
            if constexpr (VEC == 4) {
                __stcs(reinterpret_cast<float4*>(out + j0), make_float4(o[0], o[1], o[2], o[3]));
            } else {
                __stcs(out + j0, o[0]);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Workspaces

struct PassWs {
    int* err;    // k_plan_mv's error word
    float* row_part;
    float* col_part;
    void* band;  // the fallback pass's partial buffers and tickets
};

static PassWs carve_pass(void* base, const PlanOp& op, int64_t B, int64_t N, int64_t M,
                         size_t* off) {
    PassWs w{};
    char* p = (char*)base;
    auto take = [&](size_t bytes) {
        char* r = p ? p + *off : nullptr;
        *off += align_up(bytes);
        return r;
    };
    w.err = (int*)take(sizeof(int));
    w.row_part = (float*)take(sizeof(float) * B * N * op.nchunks);
    w.col_part = (float*)take(sizeof(float) * B * op.nbands * M);
    w.band = take(op.use_mv ? 0 : band_workspace_bytes(B, N, M));
    return w;
}

struct CgWs {
    CgState* st;
    double* acc;
    float *rs, *cs, *r_f, *r_g, *p_f, *p_g, *ys, *xs, *ap_f, *ap_g;
    PassWs pass;
    size_t bytes;
};

static size_t cg_state_bytes(int64_t B) { return sizeof(CgState) + sizeof(double) * 6 * B; }

static CgWs carve_cg(void* base, const PlanOp& op, int64_t B, int64_t N, int64_t M) {
    CgWs w{};
    char* p = (char*)base;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        char* r = p ? p + off : nullptr;
        off += align_up(bytes);
        return r;
    };
    const size_t fn = sizeof(float) * B * N, fm = sizeof(float) * B * M;
    w.st = (CgState*)take(cg_state_bytes(B));
    w.acc = w.st ? (double*)(w.st + 1) : nullptr;
    w.rs = (float*)take(fn);
    w.cs = (float*)take(fm);
    w.r_f = (float*)take(fn);
    w.r_g = (float*)take(fm);
    w.p_f = (float*)take(fn);
    w.p_g = (float*)take(fm);
    w.ys = (float*)take(fn);
    w.xs = (float*)take(fm);
    w.ap_f = (float*)take(fn);
    w.ap_g = (float*)take(fm);
    w.pass = carve_pass(base, op, B, N, M, &off);
    w.bytes = off;
    return w;
}

// The two layouts an operand can get (k_plan_mv's or the fallback's), so that
// the workspace size depends on B, N, M only.
static void layouts(int64_t B, int64_t N, int64_t M, PlanOp* mv, PlanOp* fb) {
    *mv = PlanOp{};
    *fb = PlanOp{};
    mv->use_mv = true;
    mv->nchunks = (M + kMvW - 1) / kMvW;
    int64_t br;
    mv->nbands = mv_bands(B, N, mv->nchunks, &br);
    fb->use_mv = false;
    fb->nchunks = fb->nbands = 1;
}

// ---------------------------------------------------------------------------
// Finished row / column sums of the P-free plan from one k_plan_mv pass, for
// the plan-side entry points (sk_plan.cu): row0 = sum_j p x_j, col0 = sum_i
// p y_i, and with `dual` also row1 = sum_j p, col1 = sum_i p.

static size_t plan_sums_parts(int64_t B, int64_t N, int64_t M, int64_t* nchunks,
                              int64_t* nbands) {
    PlanOp mv, fb;
    layouts(B, N, M, &mv, &fb);
    *nchunks = mv.nchunks;
    *nbands = mv.nbands;
    return align_up(sizeof(float) * B * N * mv.nchunks) +
           align_up(sizeof(float) * B * mv.nbands * M);
}

size_t plan_sums_bytes(int64_t B, int64_t N, int64_t M, bool dual) {
    int64_t nc, nb;
    const size_t one = plan_sums_parts(B, N, M, &nc, &nb);
    return align_up(sizeof(int)) + (dual ? 2 : 1) * one;
}

int plan_sums(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb, int64_t sCn,
              int64_t sCm, const float* f, const float* g, double epsilon,
              const uint8_t* mask_a, const uint8_t* mask_b, const float* x, const float* y,
              bool dual, float* row0, float* row1, float* col0, float* col1, void* ws,
              cudaStream_t s, bool times_c) {
    if (times_c && (dual || col0 || col1)) return kPlanSumsUnsuited;
    PlanOp op;
    if (make_op(C, B, N, M, sCb, sCn, sCm, f, g, epsilon, mask_a, mask_b, nullptr, &op) != SK_OK)
        return kPlanSumsUnsuited;
    if (!op.use_mv || (x && (uintptr_t)x % 16 != 0)) return kPlanSumsUnsuited;
    char* p = (char*)ws;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        char* r = p + off;
        off += align_up(bytes);
        return r;
    };
    int* err = (int*)take(sizeof(int));
    float* rp0 = (float*)take(sizeof(float) * B * N * op.nchunks);
    float* cp0 = (float*)take(sizeof(float) * B * op.nbands * M);
    float* rp1 = dual ? (float*)take(sizeof(float) * B * N * op.nchunks) : nullptr;
    float* cp1 = dual ? (float*)take(sizeof(float) * B * op.nbands * M) : nullptr;
    SK_CUDA(cudaMemsetAsync(err, 0, sizeof(int), s));
    if (int e = mv_smem_setup()) return e;
    MvArgs m = op.mv;
    m.x = x;
    m.y = y;
    m.row_part = rp0;
    m.col_part = (col0 || col1) ? cp0 : nullptr;
    m.row_part1 = rp1;
    m.col_part1 = cp1;
    m.skip = nullptr;
    m.err = err;
    const int64_t units = m.B * m.nbands * m.nchunks;
    const unsigned grid = (unsigned)std::min<int64_t>(units, 148 * kMvMinBlocks);
    if (dual) k_plan_mv<false, true><<<grid, kMvThreads, sizeof(MvSmem), s>>>(m);
    else if (times_c) k_plan_mv<false, false, true><<<grid, kMvThreads, sizeof(MvSmem), s>>>(m);
    else k_plan_mv<false><<<grid, kMvThreads, sizeof(MvSmem), s>>>(m);
    SK_LAUNCHED("k_plan_mv launch");
    const unsigned eg = elem_grid(B * (N + M));
    k_mv_merge<<<eg, 256, 0, s>>>(rp0, cp0, row0 ? B * N : 0, col0 ? B * M : 0, M,
                                  op.nchunks, op.nbands, row0, col0);
    if (dual)
        k_mv_merge<<<eg, 256, 0, s>>>(rp1, cp1, row1 ? B * N : 0, col1 ? B * M : 0, M,
                                      op.nchunks, op.nbands, row1, col1);
    SK_LAUNCHED("k_mv_merge launch");
    return SK_OK;
}

}  // namespace sk

using namespace sk;

extern "C" {

size_t sk_plan_matvec_workspace_bytes(int64_t B, int64_t N, int64_t M) {
    if (B <= 0 || N <= 0 || M <= 0) return 0;
    PlanOp mv, fb;
    layouts(B, N, M, &mv, &fb);
    size_t a = 0, b = 0;
    carve_pass(nullptr, mv, B, N, M, &a);
    carve_pass(nullptr, fb, B, N, M, &b);
    return std::max(a, b);
}

int sk_plan_matvec(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb, int64_t sCn,
                   int64_t sCm, const float* f, const float* g, double epsilon,
                   const uint8_t* mask_a, const uint8_t* mask_b, const float* P,
                   const float* x, const float* y, float* Px, float* Pty, float* P1,
                   float* Pt1, void* workspace, size_t workspace_bytes, void* stream) {
    clear_error();
    PlanOp op;
    if (int e = make_op(C, B, N, M, sCb, sCn, sCm, f, g, epsilon, mask_a, mask_b, P, &op))
        return e;
    if ((Px && !x) || (Pty && !y)) return fail(SK_ERR_ARG, "Px needs x and Pty needs y");
    if (!Px && !Pty && !P1 && !Pt1) return SK_OK;
    if (!workspace || workspace_bytes < sk_plan_matvec_workspace_bytes(B, N, M))
        return fail(SK_ERR_WORKSPACE, "workspace smaller than sk_plan_matvec_workspace_bytes");
    if (Px && (uintptr_t)x % 16 != 0) return fail(SK_ERR_ARG, "x must be 16-byte aligned");
    cudaStream_t s = (cudaStream_t)stream;
    size_t off = 0;
    const PassWs w = carve_pass(workspace, op, B, N, M, &off);
    SK_CUDA(cudaMemsetAsync(w.err, 0, sizeof(int), s));
    const unsigned grid = elem_grid(B * (N + M));
    if (Px || Pty) {  // weighted sums
        if (int e = run_pass(op, Px ? x : nullptr, Pty ? y : nullptr, w.row_part, w.col_part,
                             nullptr, w.err, w.band, s))
            return e;
        k_mv_merge<<<grid, 256, 0, s>>>(w.row_part, w.col_part, Px ? B * N : 0,
                                        Pty ? B * M : 0, M, op.nchunks, op.nbands, Px, Pty);
        SK_LAUNCHED("k_mv_merge launch");
    }
    if (P1 || Pt1) {  // plain sums
        if (int e = run_pass(op, nullptr, nullptr, w.row_part, w.col_part, nullptr, w.err,
                             w.band, s))
            return e;
        k_mv_merge<<<grid, 256, 0, s>>>(w.row_part, w.col_part, P1 ? B * N : 0,
                                        Pt1 ? B * M : 0, M, op.nchunks, op.nbands, P1, Pt1);
        SK_LAUNCHED("k_mv_merge launch");
    }
    return SK_OK;
}

size_t sk_implicit_workspace_bytes(int64_t B, int64_t N, int64_t M) {
    if (B <= 0 || N <= 0 || M <= 0) return 0;
    PlanOp mv, fb;
    layouts(B, N, M, &mv, &fb);
    return std::max(carve_cg(nullptr, mv, B, N, M).bytes, carve_cg(nullptr, fb, B, N, M).bytes);
}

int sk_implicit_matvec(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                       int64_t sCn, int64_t sCm, const float* f, const float* g, double epsilon,
                       const uint8_t* mask_a, const uint8_t* mask_b, const float* P,
                       const float* v_f, const float* v_g, double rho_a, double rho_b,
                       double reg, int mode, float* out_f, float* out_g, void* workspace,
                       size_t workspace_bytes, void* stream) {
    clear_error();
    PlanOp op;
    if (int e = make_op(C, B, N, M, sCb, sCn, sCm, f, g, epsilon, mask_a, mask_b, P, &op))
        return e;
    if (!v_f || !v_g || !out_f || !out_g)
        return fail(SK_ERR_ARG, "v_f, v_g, out_f and out_g must be non-NULL");
    if (mode < MV_SCHUR || mode > MV_JVP) return fail(SK_ERR_ARG, "mode must be 0, 1 or 2");
    if (!workspace || workspace_bytes < sk_implicit_workspace_bytes(B, N, M))
        return fail(SK_ERR_WORKSPACE, "workspace smaller than sk_implicit_workspace_bytes");
    cudaStream_t s = (cudaStream_t)stream;
    const CgWs w = carve_cg(workspace, op, B, N, M);
    SK_CUDA(cudaMemsetAsync(w.pass.err, 0, sizeof(int), s));
    const unsigned grid = elem_grid(B * (N + M));
    // pass 1: row and column sums r, c
    if (int e = run_pass(op, nullptr, nullptr, w.pass.row_part, w.pass.col_part, nullptr,
                         w.pass.err, w.pass.band, s))
        return e;
    k_mv_merge<<<grid, 256, 0, s>>>(w.pass.row_part, w.pass.col_part, B * N, B * M, M,
                                    op.nchunks, op.nbands, w.rs, w.cs);
    SK_LAUNCHED("k_mv_merge launch");
    const int scaled = mode != MV_JVP;
    k_mv_weights<<<elem_grid(B * N), 256, 0, s>>>(v_f, w.rs, B * N, scaled, w.ys);
    k_mv_weights<<<elem_grid(B * M), 256, 0, s>>>(v_g, w.cs, B * M, scaled, w.xs);
    SK_LAUNCHED("k_mv_weights launch");
    // pass 2: P xs and P^T ys
    if (int e = run_pass(op, w.xs, w.ys, w.pass.row_part, w.pass.col_part, nullptr,
                         w.pass.err, w.pass.band, s))
        return e;
    k_mv_merge<<<grid, 256, 0, s>>>(w.pass.row_part, w.pass.col_part, B * N, B * M, M,
                                    op.nchunks, op.nbands, w.ap_f, w.ap_g);
    SK_LAUNCHED("k_mv_merge launch");
    const float ra = (float)rho_a, rb = (float)rho_b, ca = (float)(1.0 + reg);
    // J_T^T mixes the other side's rho into the pass term; J_T its own.
    const float omr_f = (float)(mode == MV_JVP ? 1.0 - rho_a : 1.0 - rho_b);
    const float omr_g = (float)(mode == MV_JVP ? 1.0 - rho_b : 1.0 - rho_a);
    k_mv_out<<<elem_grid(B * N), 256, 0, s>>>(v_f, w.ap_f, w.rs, mask_a, B * N, mode, ra,
                                              omr_f, ca, out_f);
    k_mv_out<<<elem_grid(B * M), 256, 0, s>>>(v_g, w.ap_g, w.cs, mask_b, B * M, mode, rb,
                                              omr_g, ca, out_g);
    SK_LAUNCHED("k_mv_out launch");
    return SK_OK;
}

int sk_implicit_cg(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb, int64_t sCn,
                   int64_t sCm, const float* f, const float* g, double epsilon,
                   const uint8_t* mask_a, const uint8_t* mask_b, const float* P,
                   const float* rhs_f, const float* rhs_g, double rho_a, double rho_b,
                   int max_iters, double tol, double reg, float* lambda_f, float* lambda_g,
                   float* grad_a, float* grad_b, void* workspace, size_t workspace_bytes,
                   int* n_iters, void* stream) {
    clear_error();
    PlanOp op;
    if (int e = make_op(C, B, N, M, sCb, sCn, sCm, f, g, epsilon, mask_a, mask_b, P, &op))
        return e;
    if (!rhs_f || !rhs_g || !lambda_f || !lambda_g)
        return fail(SK_ERR_ARG, "rhs_f, rhs_g, lambda_f and lambda_g must be non-NULL");
    if (max_iters < 0) return fail(SK_ERR_ARG, "max_iters must be >= 0");
    if ((grad_a || grad_b) && !(epsilon > 0.0))
        return fail(SK_ERR_ARG, "grad_a / grad_b need epsilon > 0");
    if (!workspace || workspace_bytes < sk_implicit_workspace_bytes(B, N, M))
        return fail(SK_ERR_WORKSPACE, "workspace smaller than sk_implicit_workspace_bytes");
    cudaStream_t s = (cudaStream_t)stream;
    const CgWs w = carve_cg(workspace, op, B, N, M);
    SK_CUDA(cudaMemsetAsync(w.st, 0, cg_state_bytes(B), s));
    SK_CUDA(cudaMemsetAsync(w.pass.err, 0, sizeof(int), s));

    CgArgs c{};
    c.B = B;
    c.N = N;
    c.M = M;
    c.L = N + M;
    c.pieces = (c.L + kCgTile - 1) / kCgTile;
    c.row_part = w.pass.row_part;
    c.col_part = w.pass.col_part;
    c.nchunks = op.nchunks;
    c.nbands = op.nbands;
    c.rs = w.rs;
    c.cs = w.cs;
    c.rhs_f = rhs_f;
    c.rhs_g = rhs_g;
    c.x_f = lambda_f;
    c.x_g = lambda_g;
    c.r_f = w.r_f;
    c.r_g = w.r_g;
    c.p_f = w.p_f;
    c.p_g = w.p_g;
    c.ys = w.ys;
    c.xs = w.xs;
    c.ap_f = w.ap_f;
    c.ap_g = w.ap_g;
    c.grad_a = grad_a;
    c.grad_b = grad_b;
    c.eps = (float)epsilon;
    c.rho_a = (float)rho_a;
    c.rho_b = (float)rho_b;
    c.reg = (float)reg;
    c.tol = (float)tol;
    c.max_iters = max_iters;
    c.acc = w.acc;
    c.st = w.st;
    const unsigned grid = (unsigned)(B * c.pieces);

    // row and column sums r, c, then the start of the iteration
    if (int e = run_pass(op, nullptr, nullptr, w.pass.row_part, w.pass.col_part, nullptr,
                         w.pass.err, w.pass.band, s))
        return e;
    c.slot = 2;
    k_cg_init<<<grid, kCgThreads, 0, s>>>(c);
    SK_LAUNCHED("k_cg_init launch");
    for (int it = 0; it < max_iters; ++it) {
        // P (p_g / c) and P^T (p_f / r), then the CG update
        if (int e = run_pass(op, w.xs, w.ys, w.pass.row_part, w.pass.col_part, &w.st->done,
                             w.pass.err, w.pass.band, s))
            return e;
        c.slot = it % 3;
        k_cg_a<<<grid, kCgThreads, 0, s>>>(c);
        k_cg_b<<<grid, kCgThreads, 0, s>>>(c);
        k_cg_c<<<grid, kCgThreads, 0, s>>>(c);
        SK_LAUNCHED("k_cg launch");
    }
    if (n_iters) {
        int err = 0;
        SK_CUDA(cudaMemcpyAsync(n_iters, &w.st->n_iters, sizeof(int), cudaMemcpyDeviceToHost, s));
        SK_CUDA(cudaMemcpyAsync(&err, w.pass.err, sizeof(int), cudaMemcpyDeviceToHost, s));
        SK_CUDA(cudaStreamSynchronize(s));
        if (err) return fail(SK_ERR_TIMEOUT, "a plan pass gave up waiting for its copies");
    }
    return SK_OK;
}

int sk_implicit_dC(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb, int64_t sCn,
                   int64_t sCm, const float* f, const float* g, double epsilon,
                   const uint8_t* mask_a, const uint8_t* mask_b, const float* lambda_f,
                   const float* lambda_g, float* dC, void* stream) {
    clear_error();
    if (int e = check_problem(C, B, N, M, epsilon)) return e;
    if (!f || !g || !lambda_f || !lambda_g || !dC)
        return fail(SK_ERR_ARG, "f, g, lambda_f, lambda_g and dC must be non-NULL");
    const int64_t rows = B * N;
    const unsigned grid = (unsigned)std::min<int64_t>((rows + 7) / 8, 148 * 8);
    const BandArgs k = band_base(C, B, N, M, sCb, sCn, sCm, epsilon);  // khi, klo
    const float inv_eps = (float)(1.0 / epsilon);
    cudaStream_t s = (cudaStream_t)stream;
    if (vec4_ok(C, B, M, sCb, sCn, sCm) && (uintptr_t)dC % 16 == 0)
        k_implicit_dc<4><<<grid, 256, 0, s>>>(C, sCb, sCn, sCm, B, N, M, f, g, lambda_f,
                                             lambda_g, mask_a, mask_b, k.khi, k.klo, inv_eps,
                                             dC);
    else
        k_implicit_dc<1><<<grid, 256, 0, s>>>(C, sCb, sCn, sCm, B, N, M, f, g, lambda_f,
                                             lambda_g, mask_a, mask_b, k.khi, k.klo, inv_eps,
                                             dC);
    SK_LAUNCHED("k_implicit_dc launch");
    return SK_OK;
}

}  // extern "C"
