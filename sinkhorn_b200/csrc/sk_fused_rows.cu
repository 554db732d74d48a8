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
//     column range, R rows per stage (16 for M <= 1024, else 8; at most 64 KB),
//     into a 3-stage ring (full / empty mbarriers);
//   * 16 consumer warps. Row phase: 16 / R warps per row of the stage; their
//     lanes fold (g - c) * log2(e)/eps over the row (g staged once per launch
//     in shared memory) and reduce across the warp (and the warp pair); the
//     row's first lane forms f as the reference does (isinf guard, + eps log a,
//     rho-mix, mask) and posts the row's effective f. One named barrier.
//     Column phase: thread t folds its 4 columns over the stage's R rows with
//     the new f, one exponential per term against lazily moved references
//     (the row's max bounds its column terms, as in k_fused_iter).
// At the end every thread writes its columns' partial LSE (natural log) to
// the chunk's row of the partials, as k_fused_iter does. Exponentials run in
// log2 units (x * log2 e / eps rounded once, as in k_fused_iter) on the packed
// fp32x2 pipe. Every wait is bounded: a timeout records error 2 in the status
// record, the CTA stops waiting and lets its own copies land.
#include <algorithm>
#include <cmath>

#include "sk_common.cuh"
#include "sk_internal.h"
#include "sk_solve.cuh"
#include "sk_tma.cuh"

namespace sk {

constexpr int kRfWarps = 16;                     // consumer warps
constexpr int kRfThreads = 32 * (kRfWarps + 1);  // + the producer warp
constexpr int kRfMaxRows = 16;                   // rows per stage (M <= 1024; 8 above)
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

// Dynamic shared memory: the ring, then g, then the per-stage f and barriers.
struct RfTail {
    float fst[kRfStages][kRfMaxRows];   // effective f of the stage's rows (-inf: masked)
    float rmx[kRfStages][kRfMaxRows];   // the row's max of (g - c) log2(e)/eps
    float2 hpair[kRfMaxRows / 2][2];    // two warps per row: their (max, sum) pairs
    uint64_t full[kRfStages];
    uint64_t empty[kRfStages];
    int abort;
};

// rows per stage: 16 KB of shared memory per row slot at most
static int rf_rows(int64_t M) { return M <= 1024 ? 16 : 8; }

static size_t rf_smem_bytes(int64_t M) {
    return sizeof(float) * ((size_t)kRfStages * rf_rows(M) * M + M) + sizeof(RfTail);
}

__device__ __forceinline__ void rf_consumers_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(32 * kRfWarps) : "memory");
}

// (max, sum of 2^(x - max)) pairs in log2 units.
__device__ __forceinline__ void rf_merge(float& m, float& s, float m2, float s2) {
    const float mn = fmaxf(m, m2);
    if (mn == -INFINITY) return;
    s = s * ex2(m - mn) + s2 * ex2(m2 - mn);
    m = mn;
}

// Fold pairs of log2-unit terms into (m, s): one max pass, then one ex2 per
// term on the packed pipe and one for the rescale.
template <int K2>
__device__ __forceinline__ void rf_fold_pairs(float& m, float& s, const float2 (&x)[K2]) {
    float cm = fmaxf(x[0].x, x[0].y);
#pragma unroll
    for (int q = 1; q < K2; ++q) cm = fmaxf(cm, fmaxf(x[q].x, x[q].y));
    if (cm == -INFINITY) return;
    const float mn = fmaxf(m, cm);
    const float2 nmn = make_float2(-mn, -mn);
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int q = 0; q < K2; ++q) {
        const float2 d = __fadd2_rn(x[q], nmn);
        acc = __fadd2_rn(acc, make_float2(ex2(d.x), ex2(d.y)));
    }
    s = s * ex2(m - mn) + (acc.x + acc.y);
    m = mn;
}

__device__ __forceinline__ bool rf_wait(uint64_t* bar, uint32_t parity, volatile int* ab) {
    for (uint32_t i = 0; i < kWaitPolls; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*ab) return false;
    }
    return false;
}

// R: rows per stage (16 for M <= 1024, 8 up to 2048). WPR = 16 / R warps
// share a row in the row phase (interleaved float4 groups); with two, the pair
// meets on a 64-thread named barrier and the even warp finishes the row.
// Column phase: thread t (of 512) owns the float4 group j0 + 4 t.
template <int R>
__global__ void __launch_bounds__(kRfThreads, 1) k_rows_fused(RowsFusedArgs a) {
    constexpr int WPR = kRfWarps / R;
    pdl_wait();
    pdl_trigger();
    extern __shared__ __align__(128) unsigned char rf_smem[];
    const int64_t M = a.M;
    float* ring = reinterpret_cast<float*>(rf_smem);     // [stages][R][M]
    float* gs = ring + (size_t)kRfStages * R * M;         // [M]
    RfTail& T = *reinterpret_cast<RfTail*>(gs + M);
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
    for (int64_t j = threadIdx.x; j < M; j += kRfThreads) gs[j] = a.g_eff[b * M + j];
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
    float res = 0.f;
    const int rw = warp / WPR, hw = warp % WPR;  // row of the stage, share of it
    const int tc = threadIdx.x;                  // column group of the column phase
    const int64_t jc = j0 + 4 * tc;
    // per column: a reference cm (log2 units) and the sum of 2^(y - cm). The
    // reference moves only when a term exceeds it by more than 2^kRfLazy; a
    // row whose terms provably stay below 2^kRfFastBound of every reference
    // (its max of (g - c) k2 plus (f - g) k2 against hmin = min over this
    // thread's unmasked columns of g k2 + cm) folds without a per-element
    // check, as in k_fused_iter.
    float cm[4] = {-3.0e38f, -3.0e38f, -3.0e38f, -3.0e38f};  // finite: empty columns keep cs = 0
    float cs[4] = {0.f, 0.f, 0.f, 0.f};
    float hmin = -INFINITY;  // no bound before the first row sets the references
    // the warp's row of stage t: mask, previous f and log a, loaded one stage
    // ahead so no stage waits on them
    auto row_data = [&](int64_t t, bool& valid, float& fin, float& la) {
        const int64_t i = lr0 + t * R + rw;
        const int64_t row = b * a.N + i;
        const bool in_chunk = t < nstages && i < lr1;
        valid = in_chunk && (a.mask_a == nullptr || a.mask_a[row] != 0);
        fin = (in_chunk && lane == 0) ? a.f_in[row] : 0.f;
        la = (valid && lane == 0) ? a.log_a[row] : 0.f;
    };
    bool nvalid;
    float nfin, nla;
    row_data(0, nvalid, nfin, nla);
    for (int64_t t = 0; t < nstages; ++t) {
        const int q = (int)(t % kRfStages);
        const bool valid = nvalid;
        const float fin = nfin, la = nla;
        row_data(t + 1, nvalid, nfin, nla);
        if (!__all_sync(0xffffffffu, rf_wait(&T.full[q], (uint32_t)(t / kRfStages) & 1u, ab)))
            *ab = 1;
        const bool bad = *ab != 0;
        const float* stage = ring + (size_t)q * R * M;
        // ---- row phase: row rw of the stage, float4 groups hw*32 + lane + 32 WPR k
        const int64_t i = lr0 + t * R + rw;
        const bool in_chunk = i < lr1;
        const int64_t row = b * a.N + i;
        float m = -INFINITY, s = 0.f;
        if (valid && !bad) {
            const float* cr = stage + (size_t)rw * M;
            for (int64_t j = j0 + 4 * (hw * 32 + lane); j < j1; j += 4 * 32 * WPR * 2) {
                float2 x[4];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int64_t jj = j + 4 * 32 * WPR * h;
                    if (jj < j1) {
                        const float4 c = *reinterpret_cast<const float4*>(cr + jj);
                        const float4 g = *reinterpret_cast<const float4*>(gs + jj);
                        x[2 * h] = __fmul2_rn(
                            __ffma2_rn(make_float2(c.x, c.y), neg1, make_float2(g.x, g.y)), kk);
                        x[2 * h + 1] = __fmul2_rn(
                            __ffma2_rn(make_float2(c.z, c.w), neg1, make_float2(g.z, g.w)), kk);
                    } else {
                        x[2 * h] = x[2 * h + 1] = make_float2(-INFINITY, -INFINITY);
                    }
                }
                rf_fold_pairs<4>(m, s, x);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
                const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
                rf_merge(m, s, m2, s2);
            }
        }
        if constexpr (WPR == 2) {
            // the odd warp hands its pair to the even one
            if (hw == 1 && lane == 0) T.hpair[rw][1] = make_float2(m, s);
            asm volatile("bar.sync %0, 64;" ::"r"(2 + rw) : "memory");
            if (hw == 0 && lane == 0) {
                const float2 p = T.hpair[rw][1];
                rf_merge(m, s, p.x, p.y);
            }
        }
        if (hw == 0 && lane == 0) {
            float fe = -INFINITY;  // past the chunk's last row
            if (in_chunk) {
                float fo = 0.f;  // masked_fill(~mask_a, 0)
                if (valid) {
                    float sm = 0.f;  // an empty row gives 0
                    if (m != -INFINITY) {
                        sm = -a.eps * (kLn2 * (m + log2f(s)));
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
            T.fst[q][rw] = fe;
            T.rmx[q][rw] = m;
        }
        rf_consumers_sync();  // the stage's f values are posted
        // ---- column phase: this thread's 4 columns over the stage's R rows
        if (!bad && jc < j1) {
#pragma unroll 4
            for (int r = 0; r < R; ++r) {
                const float fr = T.fst[q][r];
                if (fr == -INFINITY) continue;
                const float4 c = *reinterpret_cast<const float4*>(stage + (size_t)r * M + jc);
                const float2 f2 = make_float2(fr, fr);
                const float2 y01 = __fmul2_rn(__ffma2_rn(make_float2(c.x, c.y), neg1, f2), kk);
                const float2 y23 = __fmul2_rn(__ffma2_rn(make_float2(c.z, c.w), neg1, f2), kk);
                if (T.rmx[q][r] + fr * k2 - hmin <= kRfFastBound) {
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
                    // references may have moved: the bound's minimum again
                    const float4 g4 = *reinterpret_cast<const float4*>(gs + jc);
                    const float gg[4] = {g4.x, g4.y, g4.z, g4.w};
                    float h = INFINITY;
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        if (gg[e] != -INFINITY) h = fminf(h, gg[e] * k2 + cm[e]);
                    hmin = h;
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&T.empty[q]);  // this warp is done with the stage
    }

    // column partials of the chunk (natural-log LSE per column): the owned
    // group from the states, the rest of the row -inf (empty)
    float* dst = a.parts + chunk * (a.B * M + 4) + b * M;
    if (jc < j1) {
        float4 o;
        o.x = cs[0] > 0.f ? kLn2 * (cm[0] + log2f(cs[0])) : -INFINITY;
        o.y = cs[1] > 0.f ? kLn2 * (cm[1] + log2f(cs[1])) : -INFINITY;
        o.z = cs[2] > 0.f ? kLn2 * (cm[2] + log2f(cs[2])) : -INFINITY;
        o.w = cs[3] > 0.f ? kLn2 * (cm[3] + log2f(cs[3])) : -INFINITY;
        *reinterpret_cast<float4*>(dst + jc) = o;
    }
    for (int64_t j = 4 * tc; j < M; j += 4 * 32 * kRfWarps)
        if (j < j0 || j >= j1)
            *reinterpret_cast<float4*>(dst + j) =
                make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    if (check) {
        res = warp_max(res);
        if (__any_sync(0xffffffffu, isnan(res))) res = NAN;
        if (lane == 0) atomic_max_nonneg(&st->res_bits, res);
    }
    if (threadIdx.x == 0 && *ab) atomicMax(&st->err, 2);
}

template <int R>
static int launch_rows_fused_t(const RowsFusedArgs& a, cudaStream_t s) {
    const size_t smem = rf_smem_bytes(a.M);
    // opt in to the largest ring once per device (every smaller size works)
    static thread_local int done[64] = {0};
    int dev = 0;
    SK_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || !done[dev]) {
        SK_CUDA(cudaFuncSetAttribute(k_rows_fused<R>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)rf_smem_bytes(R == 16 ? 1024 : kRfMaxM)));
        if (dev >= 0 && dev < 64) done[dev] = 1;
    }
    launch_pdl(k_rows_fused<R>, dim3((unsigned)(a.B * a.chunks)), dim3(kRfThreads), smem, s, a);
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
    if (rf_rows(P.M) == 16) return launch_rows_fused_t<16>(a, s);
    return launch_rows_fused_t<8>(a, s);
}

}  // namespace sk
