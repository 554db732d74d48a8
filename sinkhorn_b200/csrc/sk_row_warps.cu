// sk_row_warps.cu -- the single-read Sinkhorn iteration for rows of
// 512 < M <= 1024 columns, one row at a time per warp, with no hand-offs
// between warps.
//
// One iteration is the f-update over every row (row LSE of (g - C)/eps,
// rho-mix, mask; forward.py:14-49, 161-171) and the per-chunk column partial
// LSEs of (f_new - C)/eps for the g-update, which k_col_finish merges and
// finishes exactly as it does for the other single-read kernels. C is read
// once per iteration.
//
// A CTA owns a chunk of one batch item's valid rows (the item's valid rows
// split evenly over its chunks) over the item's valid column span. Each of
// its 8 warps takes every 8th row of the chunk, whole: lane l holds columns
// 4 (l + 32 k) .. + 3 of the span, k < 8. Each warp feeds itself: lane 0
// keeps NS rows in flight with cp.async.bulk into the warp's own ring of
// shared memory, one mbarrier per slot (every wait bounded).
//
// Per row, in log2 units (k2 = log2(e) / eps, x = (g - c) k2):
//   * the row's max m and sum s = sum 2^(x - m), kept as e = 2^(x - m) in
//     registers, then f (isinf guard, + eps log a, rho-mix, mask: the
//     reference's row update);
//   * the column fold reuses the row's exponentials: the column term is
//     2^((f - c) k2) = e * 2^(m + f k2) * 2^(-g k2), so each column keeps
//     acc = sum over rows of e * 2^(m + f k2 - H) against a per-warp pivot
//     H (moved, with acc rescaled, when a row's m + f k2 exceeds it by more
//     than 8), and its LSE is H + log2(acc) - g k2. One exponential per
//     element in all, where the two-sweep form needs two.
// A term lost to underflow in that product is below 2^-118 of 2^H; a column
// whose sum ends below 2^-72 of 2^H (a column that no row of the chunk
// reaches, far from convergence) is therefore summed again directly from C
// with its own running max, so no column loses precision.
// At the end the warps' column sums merge (pivot-aligned, in warp order)
// through shared memory and the chunk's row of the partials gets each
// column's LSE in natural-log units, as k_fused_iter writes them.
#include <algorithm>
#include <cmath>

#include "sk_common.cuh"
#include "sk_internal.h"
#include "sk_solve.cuh"
#include "sk_tma.cuh"

namespace sk {

constexpr int kRgWarps = 8;
constexpr int kRgThreads = 32 * kRgWarps;
constexpr int kRgCtasPerSm = 2;     // 128 registers per thread
constexpr int kRgK = 8;             // float4 slots per lane: 1024 columns per warp
constexpr int kRgMaxSlots = 16;     // ring slots per warp
constexpr int kRgMinM = 516, kRgMaxM = 1024;
constexpr size_t kRgRingBytes = 96 * 1024;                   // [warps][NS][WS]
constexpr size_t kRgGkBytes = kRgK * 128 * sizeof(float);    // g k2 of the span
// The pivot H moves when a row's bound m_w + f k2 exceeds it by more than
// kRgPivotLazy, so a row's factor is at most 2^kRgPivotLazy and a term lost to
// flushing (below 2^-126 before the factor) is below 2^-118 of 2^H; N of them
// stay below 2^-102 for chunks of up to 2^16 rows, 2^-30 of any column sum of
// at least kRgStarved. A smaller column sum is summed again directly.
constexpr float kRgPivotLazy = 8.f;
constexpr float kRgStarved = 0x1p-72f;

struct RowWarpsArgs {
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
    int64_t chunks;         // chunks per batch item
    int64_t rows_per_chunk; // static share of the rows outside the valid range
    int slot_floats;        // ring slot stride (multiple of 128 floats)
    int slots;              // ring slots per warp
    float k2;               // log2(e) / eps
    float eps, rho, omr;
    Status* st;
    float* lse_out;         // (B,N) the rows' LSE (natural log; -inf masked), or nullptr
    int guard;              // 1: an infinite softmin becomes 0 (the forward's guard)
};

struct RgTail {
    uint64_t full[kRgWarps][kRgMaxSlots];
    float piv[kRgWarps];  // each warp's final pivot
    int abort;
};

static size_t rg_smem_bytes() { return kRgRingBytes + kRgGkBytes + sizeof(RgTail); }

__device__ __forceinline__ bool rg_wait(uint64_t* bar, uint32_t parity, volatile int* ab) {
    for (uint32_t i = 0; i < kWaitPolls; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*ab) return false;
    }
    return false;
}

// Column j's LSE over the chunk's rows [r0, r1) straight from C (log2 units,
// running max): the fallback for a column the pivoted sums cannot resolve.
__device__ __noinline__ float rg_column_direct(const float* Cb, int64_t sCn, int64_t j,
                                               const float* f_eff, int64_t r0, int64_t r1,
                                               float k2) {
    float m = -INFINITY, s = 0.f;
    for (int64_t i = r0; i < r1; ++i) {
        const float fe = f_eff[i];
        if (fe == -INFINITY) continue;
        const float y = (fe - Cb[i * sCn + j]) * k2;
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

__global__ void __launch_bounds__(kRgThreads, kRgCtasPerSm) k_row_warps(RowWarpsArgs a) {
    constexpr int NG = kRgWarps;  // rows of the chunk taken round-robin by the warps
    constexpr int K = kRgK;
    extern __shared__ __align__(128) unsigned char rg_smem[];
    float* ring = reinterpret_cast<float*>(rg_smem);  // [warps][NS][WS]
    float* gks = reinterpret_cast<float*>(rg_smem + kRgRingBytes);  // [WS]: g k2
    RgTail& T = *reinterpret_cast<RgTail*>(rg_smem + kRgRingBytes + kRgGkBytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grp = warp;
    const int WS = a.slot_floats, NS = a.slots;
    const int64_t M = a.M, N = a.N;

    // ---- before the previous kernel has finished: only what stays constant
    // during a solve is read here (C, the valid ranges, mask_a and log a, all
    // written before the solve's first iteration), so the ring fills while the
    // previous kernel drains
    const int64_t b = blockIdx.x / a.chunks;
    const int64_t chunk = blockIdx.x % a.chunks;
    int64_t vr0 = 0, vr1 = N, c0 = 0, c1 = M;
    if (a.ranges) {
        vr0 = a.ranges[4 * b + 0];
        vr1 = a.ranges[4 * b + 1];
        c0 = a.ranges[4 * b + 2];
        c1 = a.ranges[4 * b + 3];
    }
    // the staged column span (whole float4s; columns inside it but outside
    // [c0, c1) are masked: g = -inf)
    const int64_t cw0 = c0 & ~(int64_t)3;
    const int64_t cw1 = c1 > c0 ? ((c1 + 3) & ~(int64_t)3) : cw0;
    const int kact = (int)((cw1 - cw0 + 127) / 128);  // float4 slots in use (<= K)
    const uint32_t bytes = (uint32_t)(sizeof(float) * (cw1 - cw0));
    // the chunk's valid rows, and this group's rows among them
    const int64_t nv = vr1 > vr0 ? vr1 - vr0 : 0;
    const int64_t lr0 = vr0 + nv * chunk / a.chunks;
    const int64_t lr1 = vr0 + nv * (chunk + 1) / a.chunks;
    // (a chunk's rows fit 32 bits: the row counters below are 32-bit)
    const int nt = lr1 - lr0 > grp ? (int)((lr1 - lr0 - grp + NG - 1) / NG) : 0;

    float* wring = ring + (size_t)warp * NS * WS;
    if (lane == 0) {
        for (int q = 0; q < NS; ++q) mbar_init(&T.full[warp][q], 1);
        mbar_init_fence();
    }
    if (threadIdx.x == 0) T.abort = 0;
    // slot tails past this warp's columns are never copied into: zero them
    // once (x = fma(0, -k2, -inf) = -inf there)
#pragma unroll
    for (int k = 0; k < K; ++k) {
        if (k < kact && cw0 + 4 * (lane + 32 * k) >= cw1)
            for (int q = 0; q < NS; ++q)
                *reinterpret_cast<float4*>(wring + q * WS + 4 * (lane + 32 * k)) =
                    make_float4(0.f, 0.f, 0.f, 0.f);
    }
    __syncthreads();
    volatile int* ab = &T.abort;
    const float k2 = a.k2;
    const float* Cb = a.C + b * a.sCb;
    // the first rows in flight
    const int first = nt < NS ? nt : NS;
    if (lane == 0 && bytes > 0) {
        for (int t = 0; t < first; ++t) {
            const int64_t i = lr0 + grp + NG * t;
            mbar_expect_tx(&T.full[warp][t], bytes);
            bulk_g2s(wring + t * WS, Cb + i * a.sCn + cw0, bytes, &T.full[warp][t]);
        }
    }
    int issued = bytes > 0 ? first : 0;  // rows whose copies were issued
    int landed = 0;                      // rows whose copies were waited for
    // row data, 32 rows at a time (lane l holds row 32 k + l of the group's
    // rows), the next 32 loaded while the current ones are used
    auto row_const = [&](int tt, float& la, int& fl) {
        const int64_t row = b * N + lr0 + grp + NG * tt;
        const bool valid = tt < nt && (a.mask_a == nullptr || a.mask_a[row] != 0);
        la = valid ? a.log_a[row] : 0.f;
        fl = valid ? 1 : 0;
    };
    auto row_f = [&](int tt) {
        return tt < nt ? a.f_in[b * N + lr0 + grp + NG * tt] : 0.f;
    };
    float cur_la, nxt_la;
    int cur_fl, nxt_fl;
    row_const(lane, cur_la, cur_fl);
    row_const(32 + lane, nxt_la, nxt_fl);

    // ---- the previous kernel's results (f, g, the status) from here on
    pdl_wait();
    pdl_trigger();
    Status* st = a.st;
    if (read_volatile(&st->done)) {
        // the solve is over: let the copies issued land (bounded), then leave
        if (lane == 0)
            for (int u = 0; u < issued; ++u) mbar_wait(&T.full[warp][u], 0u);
        return;
    }
    const bool check = is_check_iter(st, read_volatile(&st->iter));
    // g k2 of the span (-inf past it and at masked columns)
    for (int u = threadIdx.x; u < WS; u += kRgThreads) {
        const int64_t j = cw0 + u;
        gks[u] = j < cw1 ? a.g_eff[b * M + j] * k2 : -INFINITY;
    }
    // rows of the chunk's static share outside the valid range are masked:
    // f = 0, and their step |0 - f_prev| counts in the residual
    float res = 0.f;
    {
        const int64_t r0 = chunk * a.rows_per_chunk;
        const int64_t r1 = std::min<int64_t>(N, r0 + a.rows_per_chunk);
        for (int64_t i = r0 + threadIdx.x; i < r1; i += kRgThreads) {
            if (i >= vr0 && i < vr1) continue;
            const int64_t row = b * N + i;
            const float d = fabsf(a.f_in[row]);  // read before f_out (may alias) is written
            res = (d > res || isnan(d)) ? d : res;
            a.f_out[row] = 0.f;
            a.f_eff[row] = -INFINITY;
        }
    }
    if (b == 0 && threadIdx.x == 0) a.parts[chunk * (a.B * M + 4) + a.B * M] = 0.f;
    float cur_fin = row_f(lane), nxt_fin = row_f(32 + lane);
    __syncthreads();  // gks

    float2 acc[K][2];
#pragma unroll
    for (int k = 0; k < K; ++k) acc[k][0] = acc[k][1] = make_float2(0.f, 0.f);
    float H = -INFINITY;  // the warp's pivot (log2 units)
    const float2 nk2 = make_float2(-k2, -k2);
    const float* gsl = gks + 4 * lane;
    float fbuf = 0.f;     // f of row 32 k + lane, stored once the 32 rows are done
    float lbuf = 0.f;     // and its LSE
    int q = 0;            // ring slot of row t
    uint32_t ph = 0u;     // its phase parity, (t / NS) & 1
    int t = 0;
    for (; t < nt; ++t) {
        if ((t & 31) == 0 && t > 0) {
            cur_fin = nxt_fin;
            cur_la = nxt_la;
            cur_fl = nxt_fl;
            row_const(t + 32 + lane, nxt_la, nxt_fl);
            nxt_fin = row_f(t + 32 + lane);
        }
        const int src = t & 31;
        const float fin = __shfl_sync(0xffffffffu, cur_fin, src);
        const float la = __shfl_sync(0xffffffffu, cur_la, src);
        const bool valid = __shfl_sync(0xffffffffu, cur_fl, src) != 0;
        float2 e[K][2];
        float m = -INFINITY;
        if (bytes > 0) {
            if (!__all_sync(0xffffffffu, rg_wait(&T.full[warp][q], ph, ab))) {
                if (lane == 0) {
                    *ab = 1;
                    atomicMax(&st->err, 2);
                }
                break;
            }
            landed = t + 1;
            const float* slot = wring + q * WS + 4 * lane;
#pragma unroll
            for (int k = 0; k < K; ++k) {
                if (k < kact) {
                    const float4 c = *reinterpret_cast<const float4*>(slot + 128 * k);
                    const float4 g4 = *reinterpret_cast<const float4*>(gsl + 128 * k);
                    e[k][0] = __ffma2_rn(make_float2(c.x, c.y), nk2, make_float2(g4.x, g4.y));
                    e[k][1] = __ffma2_rn(make_float2(c.z, c.w), nk2, make_float2(g4.z, g4.w));
                    m = fmaxf(m, fmaxf(fmaxf(e[k][0].x, e[k][0].y), fmaxf(e[k][1].x, e[k][1].y)));
                }
            }
            m = warp_max(m);
            // every lane's values are in registers (they fed m): refill the slot
            __syncwarp();
            if (t + NS < nt) {
                if (lane == 0) {
                    const int64_t i = lr0 + grp + NG * (t + NS);
                    mbar_expect_tx(&T.full[warp][q], bytes);
                    bulk_g2s(wring + q * WS, Cb + i * a.sCn + cw0, bytes, &T.full[warp][q]);
                }
                issued = t + NS + 1;
            }
            if (++q == NS) {
                q = 0;
                ph ^= 1u;
            }
        }
        float s = 0.f;
        if (m != -INFINITY) {
            const float2 nm = make_float2(-m, -m);
            float2 sp = make_float2(0.f, 0.f);
#pragma unroll
            for (int k = 0; k < K; ++k) {
                if (k < kact) {
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const float2 d = __fadd2_rn(e[k][h], nm);
                        e[k][h] = make_float2(ex2(d.x), ex2(d.y));
                        sp = __fadd2_rn(sp, e[k][h]);
                    }
                }
            }
            s = warp_sum(sp.x + sp.y);
        }
        // f of the row, as the reference forms it
        float fo = 0.f;  // masked_fill(~mask_a, 0)
        if (valid) {
            float sm = 0.f;  // an empty row gives 0
            if (m != -INFINITY) {
                sm = -a.eps * (kLn2 * (m + log2f(s)));
                if (a.guard && isinf(sm)) sm = 0.f;  // isinf guard (forward.py:41)
            }
            const float full = sm + a.eps * la;
            fo = (a.rho == 0.f) ? full : a.rho * fin + a.omr * full;
        }
        if (lane == src) {
            fbuf = valid ? fo : -INFINITY;
            lbuf = (valid && m != -INFINITY) ? kLn2 * (m + log2f(s)) : -INFINITY;
        }
        if ((src == 31 || t + 1 == nt) && lane <= src) {
            // the warp's last 32 rows at once (f of a masked row is 0)
            const int64_t row = b * N + lr0 + grp + NG * (t - src + lane);
            a.f_out[row] = fbuf == -INFINITY ? 0.f : fbuf;
            a.f_eff[row] = fbuf;
            if (a.lse_out) a.lse_out[row] = lbuf;
        }
        const float d = fabsf(fo - fin);
        res = (d > res || isnan(d)) ? d : res;
        // the column fold of the row's exponentials: a term is
        // e * 2^(m + f k2 - H) in the columns' units against the pivot
        if (valid && m != -INFINITY) {
            const float rb = m + fo * k2;  // bound of the row's terms
            if (!(rb <= H + kRgPivotLazy)) {
                const float sc = ex2(H - rb);  // 0 while no row has been folded
                const float2 sc2 = make_float2(sc, sc);
#pragma unroll
                for (int k = 0; k < K; ++k) {
                    if (k < kact) {
                        acc[k][0] = __fmul2_rn(acc[k][0], sc2);
                        acc[k][1] = __fmul2_rn(acc[k][1], sc2);
                    }
                }
                H = rb;
            }
            const float F = ex2(rb - H);
            const float2 F2 = make_float2(F, F);
#pragma unroll
            for (int k = 0; k < K; ++k) {
                if (k < kact) {
                    acc[k][0] = __ffma2_rn(e[k][0], F2, acc[k][0]);
                    acc[k][1] = __ffma2_rn(e[k][1], F2, acc[k][1]);
                }
            }
        }
    }
    // after a wait gave up, this warp's copies in flight land before the CTA
    // moves on (bounded waits)
    if (lane == 0)
        for (int u = landed; u < issued; ++u)
            mbar_wait(&T.full[warp][u % NS], (uint32_t)(u / NS) & 1u);
    if (check) {
        res = warp_max(res);
        if (__any_sync(0xffffffffu, isnan(res))) res = NAN;
        if (lane == 0) atomic_max_nonneg(&st->res_bits, res);
    }

    // ---- the warps' column sums merge through the (now idle) ring
    __syncthreads();
    const bool bad = *ab != 0;
    float* scr = ring;  // [warp][WS]
#pragma unroll
    for (int k = 0; k < K; ++k)
        if (k < kact)
            *reinterpret_cast<float4*>(scr + warp * WS + 4 * (lane + 32 * k)) =
                make_float4(acc[k][0].x, acc[k][0].y, acc[k][1].x, acc[k][1].y);
    if (lane == 0) T.piv[warp] = H;
    __syncthreads();
    float* dst = a.parts + chunk * (a.B * M + 4) + b * M;
    if (!bad) {
        float hs = -INFINITY;  // the common pivot
#pragma unroll
        for (int r = 0; r < NG; ++r) hs = fmaxf(hs, T.piv[r]);
        for (int64_t j = cw0 + threadIdx.x; j < cw1; j += kRgThreads) {
            const int o = (int)(j - cw0);
            float sum = 0.f;
            if (hs != -INFINITY) {
#pragma unroll
                for (int r = 0; r < NG; ++r) {
                    const float h = T.piv[r];
                    if (h != -INFINITY) sum = fmaf(scr[r * WS + o], ex2(h - hs), sum);
                }
            }
            const float gk2 = gks[o];
            float out = -INFINITY;  // a masked column, or no valid row in the chunk
            if (gk2 != -INFINITY && hs != -INFINITY) {
                if (!(sum < kRgStarved))
                    out = kLn2 * (hs + log2f(sum) - gk2);
                else
                    out = kLn2 * rg_column_direct(Cb, a.sCn, j, a.f_eff + b * N, lr0, lr1, k2);
            }
            dst[j] = out;
        }
    }
    for (int64_t j = threadIdx.x; j < M; j += kRgThreads)
        if (j < cw0 || j >= cw1) dst[j] = -INFINITY;
}

bool row_warps_shape(int64_t N, int64_t M) {
    return M % 4 == 0 && M >= kRgMinM && M <= kRgMaxM && N >= 1;
}

// Chunks per item: about two waves of CTAs over the batch (two CTAs per SM),
// chunks at least 64 rows deep. Each CTA's first rows are already in flight
// before the previous kernel ends, so short chunks cost little; more of them
// even out items whose masks leave them different amounts of work.
int64_t row_warps_chunks(int64_t B, int64_t N) {
    const int64_t target = (2 * 148 * kRgCtasPerSm + B - 1) / B;
    return std::max<int64_t>(1, std::min<int64_t>(target, (N + 63) / 64));
}

int64_t row_warps_max_chunks(int64_t B, int64_t N) { return row_warps_chunks(B, N); }

int launch_row_warps(const Problem& P, const SweepPlan& p, const SolveWs& w, const Scalars& sc,
                      const uint8_t* mask_a, float* f, cudaStream_t s, const StepOut* out) {
    RowWarpsArgs a{};
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
    // a ring slot holds a whole row of the span, in float4 slots of the warp
    a.slot_floats = (int)(128 * ((P.M + 127) / 128));
    a.slots = (int)std::min<int64_t>(kRgMaxSlots,
                                     kRgRingBytes / (sizeof(float) * kRgWarps * a.slot_floats));
    const size_t smem = rg_smem_bytes();
    static thread_local int done[64] = {0};
    int dev = 0;
    SK_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || !done[dev]) {
        SK_CUDA(cudaFuncSetAttribute(k_row_warps, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem));
        if (dev >= 0 && dev < 64) done[dev] = 1;
    }
    launch_pdl(k_row_warps, dim3((unsigned)(a.B * a.chunks)), dim3(kRgThreads), smem, s, a);
    SK_LAUNCHED("k_row_warps launch");
    return SK_OK;
}

}  // namespace sk
