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
// width. Warps:
//   * producer (warp 16): one cp.async.bulk per row of the item's valid
//     column span, R = 8 TPC rows per stage (64 KB), into a 3-stage ring (full
//     / empty mbarriers);
//   * 16 consumer warps, 512 threads. Thread t owns the float4 column group
//     t % G (G = 512 / TPC groups, 2048 / TPC columns) for the 8 rows of row
//     set t / G of every stage: it takes those 8 x 4 values of C from shared
//     memory into registers once (and releases the stage at once), forms its
//     8 row partials (max, sum) of (g - c) log2(e)/eps, and the warp reduces
//     the 8 rows together with a halving butterfly (9 pair merges). One
//     barrier; the row's finisher thread merges the warps' partials, forms f
//     as the reference does (isinf guard, + eps log a, rho-mix, mask) and
//     posts it with the row's max. A second barrier; then each thread folds
//     its 4 columns over its 8 rows from the same registers, one exponential
//     per term against lazily moved column references (the row's max bounds
//     its column terms, as in k_fused_iter).
// At the end the TPC row sets' column states merge, and the chunk's row of
// the partials gets each column's LSE (natural log), as k_fused_iter writes
// them. Exponentials run in log2 units (x * log2 e / eps rounded once, as in
// k_fused_iter), on the packed fp32x2 pipe where the data pairs up. Every
// wait is bounded: a timeout records error 2 in the status record, the CTA
// stops waiting and lets its own copies land.
#include <algorithm>
#include <cmath>

#include "sk_common.cuh"
#include "sk_internal.h"
#include "sk_solve.cuh"
#include "sk_tma.cuh"

namespace sk {

constexpr int kRfWarps = 16;                     // consumer warps
constexpr int kRfConsumers = 32 * kRfWarps;      // 512 consumer threads
constexpr int kRfThreads = kRfConsumers + 32;    // + the producer warp
constexpr int kRfMaxRows = 32;                   // rows per stage (TPC = 4)
constexpr int kRfStages = 3;
constexpr int kRfMinM = 512, kRfMaxM = 2048;
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
};

// Shared memory after the ring.
struct RfTail {
    float fst[kRfMaxRows];          // effective f of the stage's rows (-inf: none)
    float rmx[kRfMaxRows];          // the row's max of (g - c) log2(e)/eps
    float2 wp[kRfWarps][8];         // warps' (max, sum) partials of their row set
    uint64_t full[kRfStages];
    uint64_t empty[kRfStages];
    int abort;
};

// threads per column group: 1 up to M = 2048, 2 up to 1024, 4 up to 512
static int rf_tpc(int64_t M) { return M <= 512 ? 4 : (M <= 1024 ? 2 : 1); }

static size_t rf_smem_bytes(int64_t M) {
    return sizeof(float) * (size_t)kRfStages * 8 * rf_tpc(M) * M + sizeof(RfTail);
}

__device__ __forceinline__ void rf_consumers_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kRfConsumers) : "memory");
}

// (max, sum of 2^(x - max)) pairs in log2 units.
__device__ __forceinline__ void rf_merge(float& m, float& s, float m2, float s2) {
    const float mn = fmaxf(m, m2);
    if (mn == -INFINITY) return;
    s = s * ex2(m - mn) + s2 * ex2(m2 - mn);
    m = mn;
}

__device__ __forceinline__ bool rf_wait(uint64_t* bar, uint32_t parity, volatile int* ab) {
    for (uint32_t i = 0; i < kWaitPolls; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*ab) return false;
    }
    return false;
}

// One butterfly stage of the transposed reduction: lanes whose `bit` is set
// keep the upper half of their n pairs and send the lower half across `off`.
template <int n>
__device__ __forceinline__ void rf_halve(const float (&m)[2 * n], const float (&s)[2 * n],
                                         float (&om)[n], float (&os)[n], bool hi, int off) {
#pragma unroll
    for (int i = 0; i < n; ++i) {
        const float km = hi ? m[i + n] : m[i], ks = hi ? s[i + n] : s[i];
        const float sm = hi ? m[i] : m[i + n], ss = hi ? s[i] : s[i + n];
        const float rm = __shfl_xor_sync(0xffffffffu, sm, off);
        const float rs = __shfl_xor_sync(0xffffffffu, ss, off);
        om[i] = km;
        os[i] = ks;
        rf_merge(om[i], os[i], rm, rs);
    }
}

template <int TPC>
__global__ void __launch_bounds__(kRfThreads, 1) k_rows_fused(RowsFusedArgs a) {
    constexpr int R = 8 * TPC;                 // rows per stage
    constexpr int G = kRfConsumers / TPC;      // column groups per row set
    constexpr int WPS = kRfWarps / TPC;        // warps per row set
    pdl_wait();
    pdl_trigger();
    extern __shared__ __align__(128) unsigned char rf_smem[];
    const int64_t M = a.M;
    float* ring = reinterpret_cast<float*>(rf_smem);  // [stages][R][M]
    RfTail& T = *reinterpret_cast<RfTail*>(ring + (size_t)kRfStages * R * M);
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
        for (int q = 0; q < kRfStages; ++q) {
            mbar_init(&T.full[q], 1);
            mbar_init(&T.empty[q], kRfWarps);
        }
        T.abort = 0;
        mbar_init_fence();
    }
    // rows of the chunk outside the valid range are masked: f = 0
    for (int64_t i = r0 + threadIdx.x; i < r1; i += kRfThreads) {
        if (i >= lr0 && i < lr1) continue;
        const int64_t row = b * a.N + i;
        a.f_out[row] = 0.f;
        a.f_eff[row] = -INFINITY;
    }
    if (b == 0 && threadIdx.x == 0) a.parts[chunk * (a.B * M + 4) + a.B * M] = 0.f;
    __syncthreads();
    volatile int* ab = &T.abort;

    if (warp == kRfWarps) {
        // ---- producer -----------------------------------------------------
        const uint32_t bytes = (uint32_t)(sizeof(float) * (j1 - j0));
        const float* Cb = a.C + b * a.sCb;
        int64_t t = 0;
        for (; t < nstages; ++t) {
            const int q = (int)(t % kRfStages);
            if (t >= kRfStages &&
                !__all_sync(0xffffffffu,
                            rf_wait(&T.empty[q], (uint32_t)(t / kRfStages - 1) & 1u, ab)))
                break;
            const int64_t i = lr0 + t * R + lane;
            const bool live = lane < R && i < lr1 && bytes > 0;
            const unsigned n = __popc(__ballot_sync(0xffffffffu, live));
            if (lane == 0) mbar_expect_tx(&T.full[q], n * bytes);
            __syncwarp();
            if (live)
                bulk_g2s(ring + ((size_t)q * R + lane) * M + j0, Cb + i * a.sCn + j0, bytes,
                         &T.full[q]);
        }
        // every copy issued has landed before the CTA can leave (bounded)
        const int64_t first = t > kRfStages ? t - kRfStages : 0;
        for (int64_t u = first; u < t; ++u)
            if (!rf_wait(&T.full[u % kRfStages], (uint32_t)(u / kRfStages) & 1u, ab)) *ab = 1;
        return;
    }

    // ---- consumers ---------------------------------------------------------
    const float k2 = a.k2;
    const float2 kk = make_float2(k2, k2), neg1 = make_float2(-1.f, -1.f);
    const int tc = threadIdx.x;
    const int rs = tc / G;                      // row set: rows 8 rs .. 8 rs + 7
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
    // per column: a reference cm (log2 units) and the sum of 2^(y - cm); the
    // reference moves only when a term exceeds it by more than 2^kRfLazy, and
    // a row whose terms provably stay below 2^kRfFastBound of every reference
    // (its max of (g - c) k2 plus (f - g) k2 against hmin = min over this
    // thread's unmasked columns of g k2 + cm) folds without a per-element check
    float cm[4] = {-3.0e38f, -3.0e38f, -3.0e38f, -3.0e38f};  // finite: empty columns keep cs = 0
    float cs[4] = {0.f, 0.f, 0.f, 0.f};
    float hmin = -INFINITY;  // no bound before the first row sets the references
    float res = 0.f;
    // finisher threads (tc < R): their row's mask, previous f and log a, one stage ahead
    auto row_data = [&](int64_t t, bool& in_chunk, bool& valid, float& fin, float& la) {
        const int64_t i = lr0 + t * R + tc;
        const int64_t row = b * a.N + i;
        in_chunk = tc < R && t < nstages && i < lr1;
        valid = in_chunk && (a.mask_a == nullptr || a.mask_a[row] != 0);
        fin = in_chunk ? a.f_in[row] : 0.f;
        la = valid ? a.log_a[row] : 0.f;
    };
    bool n_in, n_valid;
    float n_fin, n_la;
    row_data(0, n_in, n_valid, n_fin, n_la);
    for (int64_t t = 0; t < nstages; ++t) {
        const int q = (int)(t % kRfStages);
        const bool in_chunk = n_in, valid = n_valid;
        const float fin = n_fin, la = n_la;
        row_data(t + 1, n_in, n_valid, n_fin, n_la);
        if (!__all_sync(0xffffffffu, rf_wait(&T.full[q], (uint32_t)(t / kRfStages) & 1u, ab)))
            *ab = 1;
        const bool bad = *ab != 0;
        // this thread's 8 x 4 values of the stage, then the stage is free
        float4 c[8];
        const float* stage = ring + (size_t)q * R * M;
#pragma unroll
        for (int k = 0; k < 8; ++k)
            c[k] = (cols && !bad) ? *reinterpret_cast<const float4*>(stage + (size_t)(8 * rs + k) * M + jc)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
        __syncwarp();
        if (lane == 0) mbar_arrive(&T.empty[q]);
        // ---- row partials of the 8 rows over this thread's 4 columns
        float pm[8], ps[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float2 x01 = __fmul2_rn(__ffma2_rn(make_float2(c[k].x, c[k].y), neg1, g01), kk);
            const float2 x23 = __fmul2_rn(__ffma2_rn(make_float2(c[k].z, c[k].w), neg1, g23), kk);
            const float mx = fmaxf(fmaxf(x01.x, x01.y), fmaxf(x23.x, x23.y));
            pm[k] = mx;
            ps[k] = 0.f;
            if (mx != -INFINITY) {
                const float2 nm = make_float2(-mx, -mx);
                const float2 d01 = __fadd2_rn(x01, nm), d23 = __fadd2_rn(x23, nm);
                const float2 e = __fadd2_rn(make_float2(ex2(d01.x), ex2(d01.y)),
                                            make_float2(ex2(d23.x), ex2(d23.y)));
                ps[k] = e.x + e.y;
            }
        }
        // transposed warp reduction: lane 4 r ends with row r's warp partial
        {
            float am[4], as[4], bm[2], bs[2], cm1[1], cs1[1];
            rf_halve<4>(pm, ps, am, as, (lane & 16) != 0, 16);
            rf_halve<2>(am, as, bm, bs, (lane & 8) != 0, 8);
            rf_halve<1>(bm, bs, cm1, cs1, (lane & 4) != 0, 4);
            float m = cm1[0], s2 = cs1[0];
#pragma unroll
            for (int o = 2; o > 0; o >>= 1) {
                const float om = __shfl_xor_sync(0xffffffffu, m, o);
                const float os = __shfl_xor_sync(0xffffffffu, s2, o);
                rf_merge(m, s2, om, os);
            }
            if ((lane & 3) == 0) T.wp[warp][lane >> 2] = make_float2(m, s2);
        }
        rf_consumers_sync();  // the warps' row partials are posted
        // ---- finisher: thread r merges row r's warp partials, forms f
        if (tc < R) {
            const int rset = tc / 8, k = tc % 8;
            float m = -INFINITY, s2 = 0.f;
#pragma unroll
            for (int w = 0; w < WPS; ++w) {
                const float2 p = T.wp[rset * WPS + w][k];
                rf_merge(m, s2, p.x, p.y);
            }
            float fe = -INFINITY;  // past the chunk's last row
            if (in_chunk) {
                const int64_t row = b * a.N + lr0 + t * R + tc;
                float fo = 0.f;  // masked_fill(~mask_a, 0)
                if (valid) {
                    float sm = 0.f;  // an empty row gives 0
                    if (m != -INFINITY) {
                        sm = -a.eps * (kLn2 * (m + log2f(s2)));
                        if (isinf(sm)) sm = 0.f;  // isinf guard (forward.py:41)
                    }
                    const float full = sm + a.eps * la;
                    fo = (a.rho == 0.f) ? full : a.rho * fin + a.omr * full;
                }
                a.f_out[row] = fo;
                fe = valid ? fo : -INFINITY;
                a.f_eff[row] = fe;
                const float d = fabsf(fo - fin);
                res = (d > res || isnan(d)) ? d : res;
            }
            T.fst[tc] = fe;
            T.rmx[tc] = m;
        }
        rf_consumers_sync();  // the stage's f values are posted
        // ---- column phase: this thread's 4 columns over its 8 rows
        if (cols && !bad) {
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float fr = T.fst[8 * rs + k];
                if (fr == -INFINITY) continue;
                const float2 f2 = make_float2(fr, fr);
                const float2 y01 =
                    __fmul2_rn(__ffma2_rn(make_float2(c[k].x, c[k].y), neg1, f2), kk);
                const float2 y23 =
                    __fmul2_rn(__ffma2_rn(make_float2(c[k].z, c[k].w), neg1, f2), kk);
                if (T.rmx[8 * rs + k] + fr * k2 - hmin <= kRfFastBound) {
                    const float2 d01 = __ffma2_rn(make_float2(cm[0], cm[1]), neg1, y01);
                    const float2 d23 = __ffma2_rn(make_float2(cm[2], cm[3]), neg1, y23);
                    const float2 s01 = __fadd2_rn(make_float2(cs[0], cs[1]),
                                                  make_float2(ex2(d01.x), ex2(d01.y)));
                    const float2 s23 = __fadd2_rn(make_float2(cs[2], cs[3]),
                                                  make_float2(ex2(d23.x), ex2(d23.y)));
                    cs[0] = s01.x;
                    cs[1] = s01.y;
                    cs[2] = s23.x;
                    cs[3] = s23.y;
                } else {
                    const float y[4] = {y01.x, y01.y, y23.x, y23.y};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        // a term far above its column's reference (and the
                        // first row of every column) moves the reference to it
                        const float d = y[e] - cm[e];
                        if (d > kRfLazy) {
                            cs[e] = fmaf(cs[e], ex2(-d), 1.f);
                            cm[e] = y[e];
                        } else {
                            cs[e] += ex2(d);
                        }
                    }
                    float h = INFINITY;  // references may have moved: the bound's minimum again
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        if (gj[e] != -INFINITY) h = fminf(h, gj[e] * k2 + cm[e]);
                    hmin = h;
                }
            }
        }
    }

    // the row sets' column states merge (through the ring, now idle), then
    // the chunk's row of the partials: each column's LSE (natural log)
    if constexpr (TPC > 1) {
        rf_consumers_sync();  // every thread is past its last stage
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
    if (check && warp == 0) {  // the finisher threads are in warp 0
        res = warp_max(res);
        if (__any_sync(0xffffffffu, isnan(res))) res = NAN;
        if (lane == 0) atomic_max_nonneg(&st->res_bits, res);
    }
    if (threadIdx.x == 0 && *ab) atomicMax(&st->err, 2);
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

// Chunks per item: whole waves of one CTA per SM (the ring takes most of an
// SM's shared memory at M = 2048), chunks at least 2 stages deep.
// Chunks per item: one CTA per SM; up to four waves of chunks at least 32
// rows deep, the most waves among the best-filled ones (shorter chunks balance
// items whose masks leave them different numbers of valid rows).
int64_t rows_fused_chunks(int64_t B, int64_t N) {
    const int64_t A = 148;
    int64_t best_c = 1;
    double best_eff = -1.0;
    const int64_t cmax = rows_fused_max_chunks(B, N);
    for (int64_t c = 1; c <= cmax; ++c) {
        const int64_t units = B * c;
        const int64_t waves = (units + A - 1) / A;
        const double eff = (double)units / (double)(A * waves);
        if (eff > best_eff + 0.02) {  // fewest chunks among the best-filled
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
                      const Scalars& sc, const uint8_t* mask_a, float* f, cudaStream_t s) {
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
    switch (rf_tpc(P.M)) {
        case 4: return launch_rows_fused_t<4>(a, s);
        case 2: return launch_rows_fused_t<2>(a, s);
        default: return launch_rows_fused_t<1>(a, s);
    }
}

}  // namespace sk
