// sk_fused_rows.cu -- the single-read Sinkhorn iteration for rows that fit one
// CTA's shared memory with room to pipeline (512 <= M <= 2048).
//
// One iteration is the f-update over every row (row LSE of (g - C)/eps, rho-mix,
// mask; forward.py:14-49, 161-171) and the per-chunk column partial LSEs of
// (f_new - C)/eps for the g-update; k_col_finish merges the chunks' partials
// and finishes g exactly as it does for k_fused_iter. Both halves read the
// same staged rows, so C is read once per iteration instead of twice.
//
// A CTA owns a chunk of consecutive rows of one batch item, the whole row
// width. Three roles meet on mbarriers only (every wait bounded):
//   * producer (warp 16): one cp.async.bulk per row of the item's valid
//     column span, R = 8 TPC rows per stage into a 3-stage ring (64 KB a
//     stage at the longest rows of each TPC);
//   * 16 consumer warps, 512 threads. Thread t owns the float4 column group
//     t % G (G = 512 / TPC groups, 2048 / TPC columns) for the SR rows of row
//     set t / G of every stage: it takes those SR x 4 values of C from shared
//     memory into registers, sums the rows' 2^((g - c) log2(e)/eps - ref)
//     against per-row references (the rows' previous LSEs), adds them over
//     the warp with a halving butterfly and posts the warp's sums. It then
//     folds the PREVIOUS stage's tile, read again from the ring (which
//     releases the stage after the fold), into its 4 columns with that
//     stage's new f: one exponential per term against lazily moved column
//     references;
//   * finisher (warp 17; lane r owns row r of each stage): adds the warps'
//     sums, checks their range, forms f as the reference does (isinf guard,
//     + eps log a, rho-mix, mask), posts it with a bound of each row's terms,
//     and posts the references two stages ahead. It has a whole stage to do
//     so while the consumers work on the next one.
// A stage whose sums leave the range is summed again by the consumers with
// (max, sum) partials from the tile, still in the ring. At the end the TPC row
// sets' column states merge, and the chunk's row of the partials gets each
// column's LSE (natural log), as k_fused_iter writes them. Exponentials run
// in log2 units, on the packed fp32x2 pipe where the data pairs up. A wait
// that times out records error 2 in the status record; every role then stops
// waiting, and the producer lets its own copies land before the CTA exits.
#include <algorithm>
#include <cmath>

#include "sk_internal.h"
#include "sk_rows_stage.cuh"
#include "sk_solve.cuh"

namespace sk {

// Column references move lazily (terms up to 2^kRfLazy above them); a row
// bounded below 2^kRfFastBound of every reference takes the unchecked fold:
// sums stay below 2^(kRfFastBound + 24) for chunks of up to 2^24 rows.
constexpr float kRfLazy = 64.f;
constexpr float kRfFastBound = 96.f;

struct RowsFusedArgs {
    const float* C;
    int64_t sCb, sCn;
    int64_t B, N, M;
    const float* g_eff;     // (B,M) previous g, -inf at masked columns
    const float* f_in;      // (B,N)
    float* f_out;           // (B,N)
    float* f_eff;           // (B,N)
    const float* log_a;     // (B,N)
    const uint8_t* mask_a;  // (B,N) or nullptr
    const int* ranges;      // (B,4): valid rows [0],[1), columns [2],[3)
    float* parts;           // (chunks, B*M + 4) column LSE partials
    int64_t chunks;         // row chunks per batch item
    int64_t rows_per_chunk;
    float k2;               // log2(e) / eps
    float eps, rho, omr;
    Status* st;
    float* lse_out;         // (B,N) the rows' LSE (natural log; -inf masked), or nullptr
    int guard;              // 1: an infinite softmin becomes 0 (the forward's guard)
};

// The row pass sums 2^(x - ref) against a per-row reference ref = the row's
// previous LSE in log2 units, (eps log a - f_prev) log2(e)/eps. The pass is
// kept when the row's sum S lies in [2^kRfSumLo, 2^kRfSumHi]: every term is
// then below 2^kRfSumHi (no overflow), and the largest term is at least
// 2^(kRfSumLo - 11) for M <= 2048, so terms flushed below 2^-126 of ref are
// below 2^-55 of the row's max. A stage with any valid row outside the range
// (the first iterations of a far-off start, empty rows, NaN) is summed again
// with each lane's own max, from the stage, still in the ring.
constexpr float kRfSumLo = 0x1p-60f;
constexpr float kRfSumHi = 0x1p100f;

// Shared memory after the ring. Per-stage records alternate between two slots
// (stage t uses slot t & 1): a slot is rewritten for stage t + 2 only after
// every reader of stage t has passed the barrier that orders it.
struct RfTail {
    float2 nref[2][kRfMaxRows];       // (-ref, -ref): the stage's per-row references
                                      // (log2 units), paired for the packed pipe
    float2 fst[2][kRfMaxRows];        // (f, f): effective f of the stage's rows (-inf: none)
    float rbd[2][kRfMaxRows];         // bound of the row's terms: LSE (or max) + f k2
    float wsum[2][kRfWarps][8];       // warps' row sums against the references (SR each)
    float2 wp[kRfWarps][8];           // warps' (max, sum) partials of a stage summed again
    float smax[2];                    // largest row bound of the stage
    int slive[2];                     // 1: every row of the stage is folded
    int redo[2];                      // 1: the stage's rows are summed again
    uint64_t full[kRfStages];         // producer -> consumers: a stage landed
    uint64_t empty[kRfStages];        // consumer warps -> producer: a stage is folded
    uint64_t sums[2];                 // consumer warps -> finisher: row sums posted
    uint64_t fdone[2];                // finisher -> consumers: f (or the redo flag) posted
    uint64_t resum;                   // consumer warps -> finisher: (max, sum) partials posted
    uint64_t fdone2;                  // finisher -> consumers: f of a stage summed again
    uint64_t rready;                  // finisher -> consumers: first references posted
    int abort;
};

static size_t rf_smem_bytes(int64_t M) { return rf_ring_bytes(M) + sizeof(RfTail); }

// (max, sum of 2^(x - max)) pairs in log2 units.
__device__ __forceinline__ void rf_merge(float& m, float& s, float m2, float s2) {
    const float mn = fmaxf(m, m2);
    if (mn == -INFINITY) return;
    s = s * ex2(m - mn) + s2 * ex2(m2 - mn);
    m = mn;
}

// The rare path of a stage (a valid row's sum against its reference out of
// range): (max, sum) partials of the thread's SR rows (its tile of the stage,
// still in the ring at tp, M floats apart; zeros where the thread has no
// columns) against each lane's max, one warp reduction per row into wp[k].
// Out of line, so that what it needs around the call is saved there and not
// on the iteration's common path.
template <int SR>
__device__ __noinline__ void rf_resum_rows(const float* tp, int M, bool cols, float2 g01,
                                           float2 g23, float k2, float2* wp, int lane) {
    const float2 kk = make_float2(k2, k2), neg1 = make_float2(-1.f, -1.f);
#pragma unroll
    for (int k = 0; k < SR; ++k) {
        const float4 c = cols ? *reinterpret_cast<const float4*>(tp + k * M)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
        const float2 x01 = __fmul2_rn(__ffma2_rn(make_float2(c.x, c.y), neg1, g01), kk);
        const float2 x23 = __fmul2_rn(__ffma2_rn(make_float2(c.z, c.w), neg1, g23), kk);
        float m = fmaxf(fmaxf(x01.x, x01.y), fmaxf(x23.x, x23.y));
        float s2 = 0.f;
        if (m != -INFINITY) {
            const float2 nm = make_float2(-m, -m);
            const float2 d01 = __fadd2_rn(x01, nm), d23 = __fadd2_rn(x23, nm);
            const float2 e = __fadd2_rn(make_float2(ex2(d01.x), ex2(d01.y)),
                                        make_float2(ex2(d23.x), ex2(d23.y)));
            s2 = e.x + e.y;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float om = __shfl_xor_sync(0xffffffffu, m, o);
            const float os = __shfl_xor_sync(0xffffffffu, s2, o);
            rf_merge(m, s2, om, os);
        }
        if (lane == 0) wp[k] = make_float2(m, s2);
    }
}

template <int TPC>
__global__ void __launch_bounds__(kRfThreads, 1) k_rows_fused(RowsFusedArgs a) {
    constexpr int SR = rf_set_rows<TPC>();     // rows per thread and stage
    constexpr int ST = rf_stages<TPC>();       // ring stages (the same bytes for every SR)
    constexpr int R = SR * TPC;                // rows per stage
    constexpr int G = kRfConsumers / TPC;      // column groups per row set
    constexpr int WPS = kRfWarps / TPC;        // warps per row set
    pdl_wait();
    pdl_trigger();
    extern __shared__ __align__(128) unsigned char rf_smem[];
    const int64_t M = a.M;
    float* ring = reinterpret_cast<float*>(rf_smem);  // [stages][R][M]
    RfTail& T = *reinterpret_cast<RfTail*>(ring + (size_t)ST * R * M);
    Status* st = a.st;
    if (read_volatile(&st->done)) return;
    const bool check = is_check_iter(st, read_volatile(&st->iter));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const int64_t b = blockIdx.x / a.chunks;
    const int64_t chunk = blockIdx.x % a.chunks;
    const int64_t r0 = chunk * a.rows_per_chunk;
    const int64_t r1 = std::min<int64_t>(a.N, r0 + a.rows_per_chunk);
    int64_t vr0 = 0, vr1 = a.N, c0 = 0, c1 = M;
    if (a.ranges) {
        vr0 = a.ranges[4 * b + 0];
        vr1 = a.ranges[4 * b + 1];
        c0 = a.ranges[4 * b + 2];
        c1 = a.ranges[4 * b + 3];
    }
    // rows of the chunk that can be valid, and the staged column span (whole
    // float4s; columns inside it but outside [c0, c1) are masked: g = -inf)
    const int64_t lr0 = std::max(r0, vr0), lr1 = std::max(lr0, std::min(r1, vr1));
    const int64_t j0 = c0 & ~(int64_t)3;
    const int64_t j1 = c1 > c0 ? ((c1 + 3) & ~(int64_t)3) : j0;
    const int64_t nstages = (lr1 - lr0 + R - 1) / R;

    if (threadIdx.x == 0) {
        for (int q = 0; q < ST; ++q) {
            mbar_init(&T.full[q], 1);
            mbar_init(&T.empty[q], kRfWarps);
        }
        for (int q = 0; q < 2; ++q) {
            mbar_init(&T.sums[q], kRfWarps);
            mbar_init(&T.fdone[q], 1);
        }
        mbar_init(&T.resum, kRfWarps);
        mbar_init(&T.fdone2, 1);
        mbar_init(&T.rready, 1);
        T.abort = 0;
        mbar_init_fence();
    }
    // rows of the chunk outside the valid range are masked: f = 0, and their
    // step |0 - f_prev| counts in the residual (non-zero only after a warm
    // start from potentials that are non-zero at masked rows)
    float out_res = 0.f;
    for (int64_t i = r0 + threadIdx.x; i < r1; i += kRfThreads) {
        if (i >= lr0 && i < lr1) continue;
        const int64_t row = b * a.N + i;
        const float d = fabsf(a.f_in[row]);  // read before f_out (may alias) is written
        out_res = (d > out_res || isnan(d)) ? d : out_res;
        a.f_out[row] = 0.f;
        a.f_eff[row] = -INFINITY;
    }
    if (check && out_res != 0.f) atomic_max_nonneg(&st->res_bits, out_res);
    if (b == 0 && threadIdx.x == 0) a.parts[chunk * (a.B * M + 4) + a.B * M] = 0.f;
    __syncthreads();
    volatile int* ab = &T.abort;
    const float k2 = a.k2;

    if (warp == kRfProducer) {
        // ---- producer -----------------------------------------------------
        const uint32_t bytes = (uint32_t)(sizeof(float) * (j1 - j0));
        const float* Cb = a.C + b * a.sCb;
        // ring offsets fit 32 bits (6 stages x R x M <= 49,152 floats)
        const int stage_floats = R * (int)M;
        float* dst0 = ring + lane * (int)M + (int)j0;
        int q = 0;          // ring slot of stage t
        uint32_t ph = 0u;   // parity of (t / ST)
        int64_t t = 0;
        for (; t < nstages; ++t) {
            if (t >= ST &&
                !__all_sync(0xffffffffu, rf_wait(&T.empty[q], ph ^ 1u, ab)))
                break;
            const int64_t i = lr0 + t * R + lane;
            const bool live = lane < R && i < lr1 && bytes > 0;
            const unsigned n = __popc(__ballot_sync(0xffffffffu, live));
            if (lane == 0) mbar_expect_tx(&T.full[q], n * bytes);
            __syncwarp();
            if (live)
                bulk_g2s(dst0 + q * stage_floats, Cb + i * a.sCn + j0, bytes, &T.full[q]);
            if (++q == ST) {
                q = 0;
                ph ^= 1u;
            }
        }
        if (t < nstages && lane == 0) rf_abort(ab, st);
        // every copy issued has landed before the CTA can leave (bounded, and
        // not cut short by an abort)
        const int64_t first = t > ST ? t - ST : 0;
        for (int64_t u = first; u < t; ++u)
            if (!mbar_wait(&T.full[u % ST], (uint32_t)(u / ST) & 1u) && lane == 0)
                rf_abort(ab, st);
        return;
    }

    if (warp == kRfFinisher) {
        // ---- finisher: lane r < R owns row r of every stage ---------------
        // row data (flags: 1 in the chunk, 2 valid) of stages t, t+1, t+2
        auto row_load = [&](int64_t t, float& fin, float& la, int& fl) {
            const int64_t i = lr0 + t * R + lane;
            const int64_t row = b * a.N + i;
            const bool in_chunk = lane < R && t < nstages && i < lr1;
            const bool valid = in_chunk && (a.mask_a == nullptr || a.mask_a[row] != 0);
            fin = in_chunk ? a.f_in[row] : 0.f;
            la = valid ? a.log_a[row] : 0.f;
            fl = (in_chunk ? 1 : 0) | (valid ? 2 : 0);
        };
        // a row's reference: its LSE of the previous iteration in log2 units
        auto row_ref = [&](int fl, float fin, float la) {
            return (fl & 2) ? (a.eps * la - fin) * k2 : 0.f;
        };
        float res = 0.f;
        // row of stage t from its (max-or-reference, sum) pair in log2 units
        // (m = -inf: no term) and an upper bound of its (g - c) k2; returns
        // (effective f, bound + f k2)
        auto finish_row = [&](int64_t t, int sl, int fl, float fin, float la, float m, float s2,
                              float bound) {
            float fe = -INFINITY;  // past the chunk's last row
            if (fl & 1) {
                const int64_t row = b * a.N + lr0 + t * R + lane;
                float fo = 0.f;  // masked_fill(~mask_a, 0)
                if (fl & 2) {
                    float sm = 0.f;  // an empty row gives 0
                    if (m != -INFINITY) {
                        sm = -a.eps * (kLn2 * (m + log2f(s2)));
                        if (a.guard && isinf(sm)) sm = 0.f;  // isinf guard (forward.py:41)
                    }
                    const float full = sm + a.eps * la;
                    fo = (a.rho == 0.f) ? full : a.rho * fin + a.omr * full;
                }
                a.f_out[row] = fo;
                fe = (fl & 2) ? fo : -INFINITY;
                a.f_eff[row] = fe;
                if (a.lse_out)
                    a.lse_out[row] =
                        ((fl & 2) && m != -INFINITY) ? kLn2 * (m + log2f(s2)) : -INFINITY;
                const float d = fabsf(fo - fin);
                res = (d > res || isnan(d)) ? d : res;
            }
            const float rb = bound + fe * k2;  // read only where fe is finite
            T.fst[sl][lane] = make_float2(fe, fe);
            T.rbd[sl][lane] = rb;
            return make_float2(fe, rb);
        };
        // whether every row of the stage takes part in the column fold, and
        // the largest row bound (whole warp)
        auto post_stage = [&](int sl, float2 fr) {
            const bool live = lane >= R || fr.x != -INFINITY;
            const float mx = warp_max(lane < R ? fr.y : -INFINITY);
            const bool all = __all_sync(0xffffffffu, live);
            if (lane == 0) {
                T.slive[sl] = all ? 1 : 0;
                T.smax[sl] = mx;
            }
        };
        float f0, l0, f1, l1, f2, l2;
        int d0, d1, d2;
        row_load(0, f0, l0, d0);
        row_load(1, f1, l1, d1);
        row_load(2, f2, l2, d2);
        if (lane < R) {
            const float r0 = row_ref(d0, f0, l0), r1 = row_ref(d1, f1, l1);
            T.nref[0][lane] = make_float2(-r0, -r0);
            T.nref[1][lane] = make_float2(-r1, -r1);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&T.rready);
        uint32_t nredo = 0;
        for (int64_t t = 0; t < nstages; ++t) {
            const int sl = (int)(t & 1);
            if (!__all_sync(0xffffffffu, rf_wait(&T.sums[sl], (uint32_t)(t >> 1) & 1u, ab))) {
                if (lane == 0) rf_abort(ab, st);
                break;
            }
            float S = 0.f, r = 0.f;
            bool ok = true;
            if (lane < R) {
                const int rset = lane / SR, k = lane % SR;
#pragma unroll
                for (int w = 0; w < WPS; ++w) S += T.wsum[sl][rset * WPS + w][k];
                r = -T.nref[sl][lane].x;
                ok = !(d0 & 2) || (S >= kRfSumLo && S <= kRfSumHi);
            }
            const bool redo = !__all_sync(0xffffffffu, ok);
            if (!redo) {
                float2 fr = make_float2(-INFINITY, -INFINITY);
                if (lane < R) fr = finish_row(t, sl, d0, f0, l0, r, S, r + log2f(S));
                post_stage(sl, fr);
            }
            // the references of stage t + 2 (this slot's readers are done with stage t)
            if (lane < R) {
                const float r2 = row_ref(d2, f2, l2);
                T.nref[sl][lane] = make_float2(-r2, -r2);
            }
            if (lane == 0) T.redo[sl] = redo ? 1 : 0;
            __syncwarp();
            if (lane == 0) mbar_arrive(&T.fdone[sl]);
            if (redo) {
                if (!__all_sync(0xffffffffu, rf_wait(&T.resum, nredo & 1u, ab))) {
                    if (lane == 0) rf_abort(ab, st);
                    break;
                }
                float2 fr = make_float2(-INFINITY, -INFINITY);
                if (lane < R) {
                    const int rset = lane / SR, k = lane % SR;
                    float m = -INFINITY, s2 = 0.f;
#pragma unroll
                    for (int w = 0; w < WPS; ++w) {
                        const float2 p = T.wp[rset * WPS + w][k];
                        rf_merge(m, s2, p.x, p.y);
                    }
                    fr = finish_row(t, sl, d0, f0, l0, m, s2, m);
                }
                post_stage(sl, fr);
                __syncwarp();
                if (lane == 0) mbar_arrive(&T.fdone2);
                ++nredo;
            }
            f0 = f1;
            l0 = l1;
            d0 = d1;
            f1 = f2;
            l1 = l2;
            d1 = d2;
            row_load(t + 3, f2, l2, d2);
        }
        if (check) {
            res = warp_max(res);
            if (__any_sync(0xffffffffu, isnan(res))) res = NAN;
            if (lane == 0) atomic_max_nonneg(&st->res_bits, res);
        }
        return;
    }

    // ---- consumers ---------------------------------------------------------
    const float2 kk = make_float2(k2, k2), neg1 = make_float2(-1.f, -1.f);
    const int tc = threadIdx.x;
    const int rs = tc / G;                      // row set: rows SR rs .. SR rs + SR - 1
    const int64_t jc = j0 + 4 * (tc % G);       // this thread's 4 columns
    const bool cols = jc < j1;
    float gj[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    if (cols) {
        const float4 g4 = *reinterpret_cast<const float4*>(a.g_eff + b * M + jc);
        gj[0] = g4.x;
        gj[1] = g4.y;
        gj[2] = g4.z;
        gj[3] = g4.w;
    }
    const float2 g01 = make_float2(gj[0], gj[1]), g23 = make_float2(gj[2], gj[3]);
    // per column: a reference cm = -ncm (log2 units) and the sum of 2^(y - cm);
    // the reference moves only when a term exceeds it by more than 2^kRfLazy,
    // and a row whose terms provably stay below 2^kRfFastBound of every
    // reference (a bound of its (g - c) k2 plus (f - g) k2 against hmin = min
    // over this thread's unmasked columns of g k2 + cm) folds without a
    // per-element check
    float2 ncm01 = make_float2(3.0e38f, 3.0e38f), ncm23 = ncm01;  // finite: empty columns keep cs = 0
    float2 cs01 = make_float2(0.f, 0.f), cs23 = cs01;
    float hmin = -INFINITY;  // no bound before the first row sets the references
    if (!__all_sync(0xffffffffu, rf_wait(&T.rready, 0u, ab)) && lane == 0) rf_abort(ab, st);

    uint32_t nredo = 0;
    // this thread's tile in ring slot 0 (32-bit offsets, as the producer's)
    const int stage_floats = R * (int)M;
    const float* tile0 = ring + SR * rs * (int)M + (int)jc;
    int q = 0;          // ring slot of stage t
    int qp = 0;         // ring slot of the last stage taken
    uint32_t ph = 0u;   // parity of (t / ST)
#pragma unroll 2
    for (int64_t t = 0; t <= nstages; ++t) {
        float4 cc[SR];
        if (t < nstages) {
            // ---- this stage's tile (the stage stays until its fold)
            if (!__all_sync(0xffffffffu, rf_wait(&T.full[q], ph, ab)) && lane == 0)
                rf_abort(ab, st);
            const bool bad = *ab != 0;
            const float* tile = tile0 + q * stage_floats;
#pragma unroll
            for (int k = 0; k < SR; ++k)
                cc[k] = (cols && !bad) ? *reinterpret_cast<const float4*>(tile + k * (int)M)
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
            qp = q;
            if (++q == ST) {
                q = 0;
                ph ^= 1u;
            }
            // ---- row sums of its SR rows over this thread's 4 columns, against
            // the rows' references: x - ref = fma(g - c, k2, -ref)
            const int sl = (int)(t & 1);
            float ps[SR];
#pragma unroll
            for (int k = 0; k < SR; ++k) {
                const float2 nr = T.nref[sl][SR * rs + k];
                const float2 x01 =
                    __ffma2_rn(__ffma2_rn(make_float2(cc[k].x, cc[k].y), neg1, g01), kk, nr);
                const float2 x23 =
                    __ffma2_rn(__ffma2_rn(make_float2(cc[k].z, cc[k].w), neg1, g23), kk, nr);
                const float2 e = __fadd2_rn(make_float2(ex2(x01.x), ex2(x01.y)),
                                            make_float2(ex2(x23.x), ex2(x23.y)));
                ps[k] = e.x + e.y;
            }
            // transposed warp reduction: row r's warp sum lands in lane (32 / SR) r
            if constexpr (SR == 8) {
                const float s2 = rf_warp_rows8(ps, lane);
                if ((lane & 3) == 0) T.wsum[sl][warp][lane >> 2] = s2;
            } else {
                const float s2 = rf_warp_rows4(ps, lane);
                if ((lane & 7) == 0) T.wsum[sl][warp][lane >> 3] = s2;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&T.sums[sl]);
        }
        if (t > 0) {
            // ---- the previous stage: its f is posted (or it is summed again)
            const int64_t s = t - 1;
            const int sl = (int)(s & 1);
            if (!__all_sync(0xffffffffu, rf_wait(&T.fdone[sl], (uint32_t)(s >> 1) & 1u, ab)) &&
                lane == 0)
                rf_abort(ab, st);
            bool bad = *ab != 0;
            // the previous stage's tile, still in the ring (released after its fold)
            const int qf = t < nstages ? (qp == 0 ? ST - 1 : qp - 1) : qp;
            const float* tp = tile0 + qf * stage_floats;
            if (!bad && T.redo[sl]) {
                rf_resum_rows<SR>(tp, (int)M, cols, g01, g23, k2, T.wp[warp], lane);
                __syncwarp();
                if (lane == 0) mbar_arrive(&T.resum);
                if (!__all_sync(0xffffffffu, rf_wait(&T.fdone2, nredo & 1u, ab)) && lane == 0)
                    rf_abort(ab, st);
                ++nredo;
                bad = *ab != 0;
            }
            // ---- column fold of the previous stage's tile: 4 columns x SR rows
            if (cols && !bad) {
                if (T.slive[sl] && T.smax[sl] - hmin <= kRfFastBound) {
                    // every row of the stage folds, each inside the bound: no checks
#pragma unroll
                    for (int k = 0; k < SR; ++k) {
                        const float2 f2 = T.fst[sl][SR * rs + k];
                        const float4 cpk = *reinterpret_cast<const float4*>(tp + k * (int)M);
                        const float2 d01 = __ffma2_rn(
                            __ffma2_rn(make_float2(cpk.x, cpk.y), neg1, f2), kk, ncm01);
                        const float2 d23 = __ffma2_rn(
                            __ffma2_rn(make_float2(cpk.z, cpk.w), neg1, f2), kk, ncm23);
                        cs01 = __fadd2_rn(cs01, make_float2(ex2(d01.x), ex2(d01.y)));
                        cs23 = __fadd2_rn(cs23, make_float2(ex2(d23.x), ex2(d23.y)));
                    }
                } else {
#pragma unroll
                    for (int k = 0; k < SR; ++k) {
                        const float2 f2 = T.fst[sl][SR * rs + k];
                        if (f2.x == -INFINITY) continue;
                        const float4 cpk = *reinterpret_cast<const float4*>(tp + k * (int)M);
                        const float2 fc01 = __ffma2_rn(make_float2(cpk.x, cpk.y), neg1, f2);
                        const float2 fc23 = __ffma2_rn(make_float2(cpk.z, cpk.w), neg1, f2);
                        if (T.rbd[sl][SR * rs + k] - hmin <= kRfFastBound) {
                            const float2 d01 = __ffma2_rn(fc01, kk, ncm01);
                            const float2 d23 = __ffma2_rn(fc23, kk, ncm23);
                            cs01 = __fadd2_rn(cs01, make_float2(ex2(d01.x), ex2(d01.y)));
                            cs23 = __fadd2_rn(cs23, make_float2(ex2(d23.x), ex2(d23.y)));
                        } else {
                            const float2 y01 = __fmul2_rn(fc01, kk), y23 = __fmul2_rn(fc23, kk);
                            const float y[4] = {y01.x, y01.y, y23.x, y23.y};
                            float ncm[4] = {ncm01.x, ncm01.y, ncm23.x, ncm23.y};
                            float cs[4] = {cs01.x, cs01.y, cs23.x, cs23.y};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                // a term far above its column's reference (and the
                                // first row of every column) moves the reference to it
                                const float d = y[e] + ncm[e];
                                if (d > kRfLazy) {
                                    cs[e] = fmaf(cs[e], ex2(-d), 1.f);
                                    ncm[e] = -y[e];
                                } else {
                                    cs[e] += ex2(d);
                                }
                            }
                            ncm01 = make_float2(ncm[0], ncm[1]);
                            ncm23 = make_float2(ncm[2], ncm[3]);
                            cs01 = make_float2(cs[0], cs[1]);
                            cs23 = make_float2(cs[2], cs[3]);
                            float h = INFINITY;  // references may have moved: the bound's minimum again
#pragma unroll
                            for (int e = 0; e < 4; ++e)
                                if (gj[e] != -INFINITY) h = fminf(h, gj[e] * k2 - ncm[e]);
                            hmin = h;
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&T.empty[qf]);
        }
    }

    float cm[4] = {-ncm01.x, -ncm01.y, -ncm23.x, -ncm23.y};
    float cs[4] = {cs01.x, cs01.y, cs23.x, cs23.y};
    // the row sets' column states merge (through the ring, now idle), then
    // the chunk's row of the partials: each column's LSE (natural log)
    if constexpr (TPC > 1) {
        rf_consumers_sync();  // every consumer is past its last stage
        float2* scratch = reinterpret_cast<float2*>(ring);  // [TPC][G][4]
#pragma unroll
        for (int e = 0; e < 4; ++e) scratch[((size_t)rs * G + tc % G) * 4 + e] = make_float2(cm[e], cs[e]);
        rf_consumers_sync();
        if (rs == 0) {
#pragma unroll
            for (int e = 0; e < 4; ++e)
                for (int r2 = 1; r2 < TPC; ++r2) {
                    const float2 o = scratch[((size_t)r2 * G + tc) * 4 + e];
                    const float mn = fmaxf(cm[e], o.x);
                    cs[e] = cs[e] * ex2(cm[e] - mn) + o.y * ex2(o.x - mn);
                    cm[e] = mn;
                }
        }
    }
    float* dst = a.parts + chunk * (a.B * M + 4) + b * M;
    if (rs == 0 && cols) {
        float4 o;
        o.x = cs[0] > 0.f ? kLn2 * (cm[0] + log2f(cs[0])) : -INFINITY;
        o.y = cs[1] > 0.f ? kLn2 * (cm[1] + log2f(cs[1])) : -INFINITY;
        o.z = cs[2] > 0.f ? kLn2 * (cm[2] + log2f(cs[2])) : -INFINITY;
        o.w = cs[3] > 0.f ? kLn2 * (cm[3] + log2f(cs[3])) : -INFINITY;
        *reinterpret_cast<float4*>(dst + jc) = o;
    }
    for (int64_t j = 4 * tc; j < M; j += 4 * kRfConsumers)
        if (j < j0 || j >= j1)
            *reinterpret_cast<float4*>(dst + j) =
                make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
}

template <int TPC>
static int launch_rows_fused_t(const RowsFusedArgs& a, cudaStream_t s) {
    const size_t smem = rf_smem_bytes(a.M);
    // opt in to the largest ring once per device (every smaller size works)
    static thread_local int done[64] = {0};
    int dev = 0;
    SK_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || !done[dev]) {
        SK_CUDA(cudaFuncSetAttribute(k_rows_fused<TPC>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)rf_smem_bytes(2048 / TPC)));
        if (dev >= 0 && dev < 64) done[dev] = 1;
    }
    launch_pdl(k_rows_fused<TPC>, dim3((unsigned)(a.B * a.chunks)), dim3(kRfThreads), smem, s,
               a);
    SK_LAUNCHED("k_rows_fused launch");
    return SK_OK;
}

bool rows_fused_shape(int64_t N, int64_t M) {
    return M % 4 == 0 && M >= kRfMinM && M <= kRfMaxM && N >= 1;
}

// Chunks per item: one CTA per SM (the ring takes most of its shared memory),
// chunks at least 32 rows deep, up to four waves. Among the chunk counts the
// fewest win unless more fill the SMs at least 5% better: every wave pays a
// ring fill, while shorter chunks balance items whose masks leave them
// different numbers of valid rows.
int64_t rows_fused_chunks(int64_t B, int64_t N) {
    const int64_t A = 148;
    int64_t best_c = 1;
    double best_eff = -1.0;
    const int64_t cmax = rows_fused_max_chunks(B, N);
    for (int64_t c = 1; c <= cmax; ++c) {
        const int64_t units = B * c;
        const int64_t waves = (units + A - 1) / A;
        const double eff = (double)units / (double)(A * waves);
        if (eff > best_eff + 0.05) {  // fewest chunks among the best-filled
            best_eff = eff;
            best_c = c;
        }
    }
    return best_c;
}

int64_t rows_fused_max_chunks(int64_t B, int64_t N) {
    return std::max<int64_t>(1, std::min<int64_t>((4 * 148 + B - 1) / B, (N + 31) / 32));
}

int launch_rows_fused(const Problem& P, const SweepPlan& p, const SolveWs& w,
                      const Scalars& sc, const uint8_t* mask_a, float* f, cudaStream_t s,
                      const StepOut* out) {
    RowsFusedArgs a{};
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
    a.ranges = w.ranges;
    a.parts = w.fparts;
    a.chunks = p.chunks;
    a.rows_per_chunk = p.rows_per_chunk;
    a.k2 = (float)(1.4426950408889634074 / (double)sc.eps);
    a.eps = sc.eps;
    a.rho = sc.rho_a;
    a.omr = sc.omr_a;
    a.st = (Status*)w.status;
    a.guard = 1;
    if (out) {
        a.f_in = out->f_in;
        a.f_out = out->f_out;
        a.lse_out = out->lse_out;
        a.guard = out->guard;
    }
    switch (rf_tpc(P.M)) {
        case 4: return launch_rows_fused_t<4>(a, s);
        case 2: return launch_rows_fused_t<2>(a, s);
        default: return launch_rows_fused_t<1>(a, s);
    }
}

}  // namespace sk
