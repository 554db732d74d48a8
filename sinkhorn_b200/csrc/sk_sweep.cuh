// sk_sweep.cuh -- the two streaming sweeps of one Sinkhorn iteration.
//
// Row sweep (f-update): one row of C per group of TPR threads, 128-bit
// streaming loads, per-thread online (max, sum 2^x) folded 16 terms at a
// time, shuffle + shared-memory merge, then the fused epilogue
//   f_new = rho f + (1-rho)(softmin + eps log a), masked rows -> 0,
// the |f_new - f| residual and (for the backward) the row LSE.
// Restates _stable_lse_row_kernel + sinkhorn_row_update
// (src/sinkhorn/triton/lse_kernel.py:21-134, src/sinkhorn/triton/forward.py:14-49).
//
// Column sweep (g-update): C is row-major, so a column LSE is computed by
// tiles of 32*VEC columns x one band of rows: each warp reads whole 512-byte
// row segments, each thread keeps per-column (max, sum) pairs over 8-row
// register chunks, the 8 row lanes of the CTA merge in shared memory and the
// band's partial LSE goes to the workspace. The last CTA of a column tile
// (atomic ticket) merges the bands and applies the fused epilogue
//   g_new = rho g + (1-rho)(softmin + eps log b), masked columns -> 0,
// the |g_new - g| residual, and -- in the last tile of the iteration -- the
// convergence decision and the iteration counter.
// Restates _stable_lse_col_kernel + sinkhorn_col_update + the check of
// src/sinkhorn/triton/forward.py:52-82,161-184, without its strided loads.
#pragma once

#include "sk_common.cuh"
#include "sk_tma.cuh"

namespace sk {

struct RowArgs {
    const float* C;
    int64_t sCb, sCn, sCm;
    int64_t B, N, M;
    const float* g_eff;     // (B,M) column potentials, -inf at masked columns
    const float* f_in;      // (B,N) previous f
    float* f_out;           // (B,N) new f (may alias f_in)
    float* f_eff;           // (B,N) new f with -inf at masked rows, or nullptr
    const float* log_a;     // (B,N), or nullptr for the plain softmin
    const uint8_t* mask_a;  // (B,N) or nullptr
    const int* ranges;      // (B,4) row_lo,row_hi,col_lo,col_hi or nullptr
    float* lse_out;         // (B,N) row LSE (natural log), or nullptr
    float k;                // 1/eps
    float eps, rho, omr;
    int guard;              // isinf -> 0 on the softmin (forward semantics)
    int plain;              // 1: f_out = softmin only (lse_row)
    Status* st;             // nullptr for a standalone sweep
};

struct ColArgs {
    const float* C;
    int64_t sCb, sCn, sCm;
    int64_t B, N, M;
    const float* f_eff;     // (B,N) row potentials, -inf at masked rows
    const float* g_in;      // (B,M)
    float* g_out;           // (B,M)
    float* g_eff;           // (B,M) or nullptr
    const float* log_b;     // (B,M) or nullptr for the plain softmin
    const uint8_t* mask_b;  // (B,M) or nullptr
    const int* ranges;
    float* partial;         // (B, nbands, M) band LSEs (natural log)
    unsigned* tickets;      // (B, ntiles), zero between launches
    float* lse_out;         // (B,M) column LSE (natural log), or nullptr
    int64_t ntiles, nbands, band_rows;
    float k, eps, rho, omr;  // k = 1/eps
    int guard;
    int plain;              // 1: g_out = softmin only (lse_col)
                            // 2: g_out = column LSE of these rows only (a rank's
                            //    partial of a row-sharded problem), no update
    Status* st;
};

__device__ __forceinline__ bool is_check_iter(const Status* st, int iter) {
    return st->check_every > 0 && ((iter + 1) % st->check_every) == 0;
}

// ---------------------------------------------------------------------------
// T: element type of C (float, or uint16_t holding bf16).
template <int VEC, int TPR, typename T = float>
__global__ void __launch_bounds__(kRowThreads) k_row_sweep(RowArgs a) {
    pdl_wait();
    pdl_trigger();
    constexpr int RPC = kRowThreads / TPR;  // rows per CTA
    constexpr int WPR = TPR / 32;           // warps per row
    constexpr int NW = kRowThreads / 32;
    __shared__ float sh_m[NW], sh_s[NW], sh_res[NW];

    Status* st = a.st;
    bool check = false;
    if (st) {
        if (read_volatile(&st->done)) return;
        check = is_check_iter(st, read_volatile(&st->iter));
    }
    const int tid = threadIdx.x;
    const int slot = tid / TPR, lt = tid % TPR;
    const int64_t nrows = a.B * a.N;
    const int64_t row = (int64_t)blockIdx.x * RPC + slot;
    const bool active = row < nrows;

    float m = -INFINITY, s = 0.f;
    bool row_valid = false;
    int64_t b = 0, i = 0;
    if (active) {
        b = row / a.N;
        i = row - b * a.N;
        row_valid = (a.mask_a == nullptr) || (a.mask_a[row] != 0);
        if (row_valid) {
            int64_t lo = 0, hi = a.M;
            if (a.ranges) {
                lo = a.ranges[4 * b + 2];
                hi = a.ranges[4 * b + 3];
            }
            const T* Crow = reinterpret_cast<const T*>(a.C) + b * a.sCb + i * a.sCn;
            const float* grow = a.g_eff + b * a.M;
            const float k = a.k;
            if constexpr (VEC == 4) {
                // columns outside [lo,hi) inside the rounded range are masked
                // (g_eff = -inf), so rounding to whole float4s is harmless
                const int64_t v0 = lo >> 2, v1 = (hi + 3) >> 2;
                constexpr int U = 4;
                int64_t v = v0 + lt;
                for (; v + (U - 1) * TPR < v1; v += U * TPR) {
                    float4 c[U], gg[U];
#pragma unroll
                    for (int u = 0; u < U; ++u) {
                        c[u] = ld_c4<T>(Crow + 4 * (v + u * TPR));
                        gg[u] = ld_vec4(grow + 4 * (v + u * TPR));
                    }
                    float2 x[2 * U];  // column pairs on the packed fp32x2 pipe
#pragma unroll
                    for (int u = 0; u < U; ++u) {
                        x[2 * u + 0] = scaled_diff2(make_float2(gg[u].x, gg[u].y),
                                                    make_float2(c[u].x, c[u].y), k);
                        x[2 * u + 1] = scaled_diff2(make_float2(gg[u].z, gg[u].w),
                                                    make_float2(c[u].z, c[u].w), k);
                    }
                    lse_fold_pairs<2 * U>(m, s, x);
                }
                for (; v < v1; v += TPR) {
                    float4 c = ld_c4<T>(Crow + 4 * v);
                    float4 gg = ld_vec4(grow + 4 * v);
                    const float2 x[2] = {
                        scaled_diff2(make_float2(gg.x, gg.y), make_float2(c.x, c.y), k),
                        scaled_diff2(make_float2(gg.z, gg.w), make_float2(c.z, c.w), k)};
                    lse_fold_pairs<2>(m, s, x);
                }
            } else {
                constexpr int U = 4;
                int64_t j = lo + lt;
                for (; j + (U - 1) * TPR < hi; j += U * TPR) {
                    float x[U];
#pragma unroll
                    for (int u = 0; u < U; ++u) {
                        int64_t jj = j + u * TPR;
                        x[u] = (__ldg(grow + jj) - ld_c1<T>(Crow + jj * a.sCm)) * k;
                    }
                    lse_fold<U>(m, s, x);
                }
                for (; j < hi; j += TPR) {
                    float x[1] = {(__ldg(grow + j) - ld_c1<T>(Crow + j * a.sCm)) * k};
                    lse_fold<1>(m, s, x);
                }
            }
        }
    }

    // merge the TPR partial pairs of each row
    warp_lse_reduce(m, s);
    if constexpr (WPR > 1) {
        const int w = tid >> 5;
        if ((tid & 31) == 0) {
            sh_m[w] = m;
            sh_s[w] = s;
        }
        __syncthreads();
        if (lt == 0) {
            for (int q = 1; q < WPR; ++q) lse_merge(m, s, sh_m[w + q], sh_s[w + q]);
        }
    }

    float res = 0.f;
    if (active && lt == 0) {
        const float fin = a.f_in ? a.f_in[row] : 0.f;
        float fo;
        if (a.plain) {
            fo = softmin_from_pair(m, s, a.eps, false);
        } else if (!row_valid) {
            fo = 0.f;  // masked_fill(~mask_a, 0) (forward.py:168-169)
        } else {
            const float sm = softmin_from_pair(m, s, a.eps, a.guard != 0);
            const float full = sm + a.eps * a.log_a[row];
            fo = (a.rho == 0.f) ? full : a.rho * fin + a.omr * full;
        }
        a.f_out[row] = fo;
        if (a.f_eff) a.f_eff[row] = row_valid ? fo : -INFINITY;
        if (a.lse_out) a.lse_out[row] = lse_of(m, s);
        res = fabsf(fo - fin);
    }
    if (check) {
        res = warp_max(res);
        if ((tid & 31) == 0) sh_res[tid >> 5] = res;
        __syncthreads();
        if (tid == 0) {
            float r = sh_res[0];
            for (int q = 1; q < NW; ++q) r = fmaxf(r, sh_res[q]);
            // NaN is kept (fmaxf would drop it): any NaN row poisons the check
            for (int q = 0; q < NW; ++q)
                if (isnan(sh_res[q])) r = sh_res[q];
            atomic_max_nonneg(&st->res_bits, r);
        }
    }
}

// ---------------------------------------------------------------------------
// Tail of a column sweep, shared by the register-chunk and bulk-copy kernels:
// merge the kColRL row-lane pairs of the tile (sh_m/sh_s: [kColRL][TJ]), write
// the band partial, take the tile ticket; the last band CTA of the tile merges
// the bands and applies the epilogue, and the last tile of the iteration takes
// the convergence decision. Every thread of the CTA calls it.
template <int TJ>
__device__ __forceinline__ void col_tail(const ColArgs& a, int64_t b, int64_t tile,
                                         int64_t band, int iter, bool check,
                                         const float* sh_m, const float* sh_s,
                                         float* sh_res, int* sh_last) {
    Status* st = a.st;
    __syncthreads();
    // merge the row lanes; one thread per column of the tile
    for (int c = threadIdx.x; c < TJ; c += blockDim.x) {
        const int64_t j = tile * TJ + c;
        if (j >= a.M) continue;
        float mm = sh_m[c], ss = sh_s[c];
#pragma unroll
        for (int q = 1; q < kColRL; ++q) lse_merge(mm, ss, sh_m[q * TJ + c], sh_s[q * TJ + c]);
        a.partial[(b * a.nbands + band) * a.M + j] = lse_of(mm, ss);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(&a.tickets[b * a.ntiles + tile], 1u);
        *sh_last = (prev == (unsigned)(a.nbands - 1));
    }
    __syncthreads();
    if (!*sh_last) return;

    // ---- last band of this column tile: merge bands, update g -------------
    __threadfence();
    float res = 0.f;
    for (int c = threadIdx.x; c < TJ; c += blockDim.x) {
        const int64_t j = tile * TJ + c;
        if (j >= a.M) continue;
        const int64_t col = b * a.M + j;
        float mm = -INFINITY, ss = 0.f;
        for (int64_t q = 0; q < a.nbands; ++q) {
            const float p = __ldcg(a.partial + (b * a.nbands + q) * a.M + j);
            lse_merge(mm, ss, p, 1.f);
        }
        const float gin = a.g_in ? a.g_in[col] : 0.f;
        const bool valid = (a.mask_b == nullptr) || (a.mask_b[col] != 0);
        float go;
        if (a.plain == 2) {
            a.g_out[col] = lse_of(mm, ss);
            continue;
        } else if (a.plain) {
            go = softmin_from_pair(mm, ss, a.eps, false);
        } else if (!valid) {
            go = 0.f;  // masked_fill(~mask_b, 0) (forward.py:170-171)
        } else {
            const float sm = softmin_from_pair(mm, ss, a.eps, a.guard != 0);
            const float full = sm + a.eps * a.log_b[col];
            go = (a.rho == 0.f) ? full : a.rho * gin + a.omr * full;
        }
        a.g_out[col] = go;
        if (a.g_eff) a.g_eff[col] = valid ? go : -INFINITY;
        if (a.lse_out) a.lse_out[col] = lse_of(mm, ss);
        const float d = fabsf(go - gin);
        res = (d > res || isnan(d)) ? d : res;
    }
    if (threadIdx.x == 0) a.tickets[b * a.ntiles + tile] = 0u;
    if (a.plain == 2) {
        // the rank's f residual travels with its partial (slot B*M)
        if (b == 0 && tile == 0 && threadIdx.x == 0)
            a.g_out[a.B * a.M] = st ? __uint_as_float(atomicOr(&st->res_bits, 0u)) : 0.f;
        return;
    }
    if (!st) return;

    if (check) {
        float r = warp_max(res);
        // keep NaN visible through the shuffle max
        if (__any_sync(0xffffffffu, isnan(res))) r = NAN;
        if ((threadIdx.x & 31) == 0) sh_res[threadIdx.x >> 5] = r;
        __syncthreads();
        if (threadIdx.x == 0) {
            float rr = sh_res[0];
            for (int q = 1; q < (int)(blockDim.x >> 5); ++q)
                rr = (sh_res[q] > rr || isnan(sh_res[q])) ? sh_res[q] : rr;
            atomic_max_nonneg(&st->res_bits, rr);
        }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(&st->ticket, 1u);
        if (prev == (unsigned)(a.B * a.ntiles - 1)) {
            // every column tile of every batch item is final: close the iteration
            __threadfence();
            st->ticket = 0u;
            if (check) {
                const float r = __uint_as_float(atomicOr(&st->res_bits, 0u));
                if (st->decide && r < st->threshold) {
                    st->converged = 1;
                    st->done = 1;
                    st->n_iters = iter + 1;
                }
                // decide == 0: the host reads res_bits, then clears it
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

// ---------------------------------------------------------------------------
// Column sweep fed by the tensor-memory accelerator (float4 layouts only).
// A producer warp streams 64-row x 128-column boxes of C (32 KB, one
// cp.async.bulk.tensor.3d per stage) into a kBulkStages-deep shared-memory
// ring; the 8 consumer warps (one row lane each) fold 8 rows per stage per
// thread. Bytes in flight no longer depend on registers.
constexpr int kBulkRows = 64;    // rows per stage = 8 per row lane
constexpr int kBulkStages = 2;
constexpr int kBulkThreads = kColThreads + 32;  // 8 consumer warps + 1 producer
constexpr int kBulkStageFloats = kBulkRows * 128;
constexpr size_t kBulkSmem =
    (size_t)kBulkStages * kBulkStageFloats * sizeof(float) + 2 * kBulkStages * sizeof(uint64_t);

__device__ __forceinline__ bool mbar_wait_or_abort(uint64_t* bar, uint32_t parity,
                                                   volatile int* abort_flag) {
    for (uint32_t i = 0; i < kWaitPolls; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
    }
    return false;
}

template <int STAGES = kBulkStages>
__global__ void __launch_bounds__(kBulkThreads)
    k_col_sweep_tma(const __grid_constant__ CUtensorMap tmap, ColArgs a) {
    pdl_wait();
    pdl_trigger();
    static_assert(STAGES == kBulkStages, "ring depth is fixed by kBulkSmem");
    extern __shared__ __align__(128) unsigned char smem[];
    float* buf = reinterpret_cast<float*>(smem);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)kBulkStages * kBulkStageFloats * 4);
    uint64_t* empty = full + kBulkStages;
    __shared__ float sh_res[kBulkThreads / 32];
    __shared__ int sh_last;
    __shared__ volatile int sh_abort;

    Status* st = a.st;
    int iter = 0;
    bool check = false;
    if (st) {
        if (read_volatile(&st->done)) return;
        iter = read_volatile(&st->iter);
        check = is_check_iter(st, iter);
    }
    const int64_t cta = blockIdx.x;
    const int64_t tile = cta % a.ntiles;
    const int64_t t2 = cta / a.ntiles;
    const int64_t band = t2 % a.nbands;
    const int64_t b = t2 / a.nbands;
    int64_t r_lo = band * a.band_rows;
    int64_t r_hi = r_lo + a.band_rows < a.N ? r_lo + a.band_rows : a.N;
    int64_t c_lo = 0, c_hi = a.M;
    if (a.ranges) {
        const int64_t vlo = a.ranges[4 * b + 0], vhi = a.ranges[4 * b + 1];
        if (r_lo < vlo) r_lo = vlo;
        if (r_hi > vhi) r_hi = vhi;
        c_lo = a.ranges[4 * b + 2];
        c_hi = a.ranges[4 * b + 3];
    }
    const bool live = (r_lo < r_hi) && (tile * 128 < c_hi) && ((tile + 1) * 128 > c_lo);
    const int64_t nrows = live ? r_hi - r_lo : 0;
    const int64_t nst = (nrows + kBulkRows - 1) / kBulkRows;

    if (threadIdx.x == 0) {
        for (int q = 0; q < kBulkStages; ++q) {
            mbar_init(&full[q], 1);
            mbar_init(&empty[q], kColRL);
        }
        sh_abort = 0;
        mbar_init_fence();
    }
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float m[4], s[4];
#pragma unroll
    for (int v = 0; v < 4; ++v) {
        m[v] = -INFINITY;
        s[v] = 0.f;
    }
    if (warp == kColRL) {
        // ---- producer ---------------------------------------------------
        if (lane == 0 && nst > 0) {
            tma_prefetch_map(&tmap);
            int64_t issued = 0;
            for (int64_t t = 0; t < nst; ++t) {
                const int q = (int)(t % kBulkStages);
                if (t >= kBulkStages &&
                    !mbar_wait_or_abort(&empty[q], (uint32_t)((t / kBulkStages) - 1) & 1u,
                                        &sh_abort)) {
                    sh_abort = 1;
                    break;
                }
                mbar_expect_tx(&full[q], (uint32_t)(kBulkStageFloats * sizeof(float)));
                tma_load_3d(buf + (size_t)q * kBulkStageFloats, &tmap, (int)(tile * 128),
                            (int)(r_lo + t * kBulkRows), (int)b, &full[q]);
                issued = t + 1;
            }
            // every issued copy must land before the CTA may leave
            const int64_t first = issued > kBulkStages ? issued - kBulkStages : 0;
            for (int64_t t = first; t < issued; ++t)
                if (!mbar_wait(&full[t % kBulkStages], (uint32_t)(t / kBulkStages) & 1u))
                    sh_abort = 1;
        }
    } else {
        // ---- consumers: warp = row lane, lane = column thread ------------
        const int rl = warp, ct = lane;
        const int64_t j0 = tile * 128 + (int64_t)ct * 4;
        const bool colok = j0 < a.M;
        const float* fb = a.f_eff + b * a.N;
        const float k = a.k;
        for (int64_t t = 0; t < nst; ++t) {
            const int q = (int)(t % kBulkStages);
            if (!mbar_wait_or_abort(&full[q], (uint32_t)(t / kBulkStages) & 1u, &sh_abort)) {
                sh_abort = 1;
                break;
            }
            const int64_t rows = (nrows - t * kBulkRows) < kBulkRows ? (nrows - t * kBulkRows)
                                                                  : kBulkRows;
            const float* stage = buf + (size_t)q * kBulkStageFloats;
            float x[4][kColChunk];
#pragma unroll
            for (int u = 0; u < kColChunk; ++u) {
                const int r = rl + kColRL * u;
                float fi = -INFINITY;
                if (r < rows) fi = __ldg(fb + r_lo + t * kBulkRows + r);
                if (fi != -INFINITY && colok) {
                    const float4 c = *reinterpret_cast<const float4*>(stage + r * 128 + ct * 4);
                    const float2 f2 = make_float2(fi, fi);
                    const float2 x01 = scaled_diff2(f2, make_float2(c.x, c.y), k);
                    const float2 x23 = scaled_diff2(f2, make_float2(c.z, c.w), k);
                    x[0][u] = x01.x;
                    x[1][u] = x01.y;
                    x[2][u] = x23.x;
                    x[3][u] = x23.y;
                } else {
#pragma unroll
                    for (int v = 0; v < 4; ++v) x[v][u] = -INFINITY;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[q]);
            lse_fold_x2<kColChunk>(m[0], s[0], m[1], s[1], x[0], x[1]);
            lse_fold_x2<kColChunk>(m[2], s[2], m[3], s[3], x[2], x[3]);
        }
    }
    __syncthreads();  // every copy has landed and every stage is read
    if (sh_abort && st && threadIdx.x == 0) atomicMax(&st->err, 2);
    float* sh_m = buf;                  // [kColRL][128], reusing stage memory
    float* sh_s = buf + kColRL * 128;
    if (warp < kColRL) {
#pragma unroll
        for (int v = 0; v < 4; ++v) {
            sh_m[warp * 128 + lane * 4 + v] = m[v];
            sh_s[warp * 128 + lane * 4 + v] = s[v];
        }
    }
    col_tail<128>(a, b, tile, band, iter, check, sh_m, sh_s, sh_res, &sh_last);
}

// T: element type of C (float, or uint16_t holding bf16).
template <int VEC, typename T = float>
__global__ void __launch_bounds__(kColThreads) k_col_sweep(ColArgs a) {
    pdl_wait();
    pdl_trigger();
    constexpr int TJ = kColCT * VEC;  // columns per tile
    __shared__ float sh_m[kColRL][TJ];
    __shared__ float sh_s[kColRL][TJ];
    __shared__ float sh_res[kColThreads / 32];
    __shared__ int sh_last;

    Status* st = a.st;
    int iter = 0;
    bool check = false;
    if (st) {
        if (read_volatile(&st->done)) return;
        iter = read_volatile(&st->iter);
        check = is_check_iter(st, iter);
    }
    const int64_t cta = blockIdx.x;
    const int64_t tile = cta % a.ntiles;
    const int64_t t2 = cta / a.ntiles;
    const int64_t band = t2 % a.nbands;
    const int64_t b = t2 / a.nbands;
    const int ct = threadIdx.x % kColCT, rl = threadIdx.x / kColCT;
    const int64_t j0 = tile * TJ + (int64_t)ct * VEC;

    int64_t r_lo = band * a.band_rows;
    int64_t r_hi = r_lo + a.band_rows < a.N ? r_lo + a.band_rows : a.N;
    int64_t c_lo = 0, c_hi = a.M;
    if (a.ranges) {
        const int64_t vlo = a.ranges[4 * b + 0], vhi = a.ranges[4 * b + 1];
        if (r_lo < vlo) r_lo = vlo;
        if (r_hi > vhi) r_hi = vhi;
        c_lo = a.ranges[4 * b + 2];
        c_hi = a.ranges[4 * b + 3];
    }
    const bool live = (r_lo < r_hi) && (tile * TJ < c_hi) && ((tile + 1) * TJ > c_lo);

    float m[VEC], s[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
        m[v] = -INFINITY;
        s[v] = 0.f;
    }
    if (live && j0 < a.M) {
        const T* Cb = reinterpret_cast<const T*>(a.C) + b * a.sCb;
        const float* fb = a.f_eff + b * a.N;
        const float k = a.k;
        for (int64_t i0 = r_lo + rl; i0 < r_hi; i0 += (int64_t)kColRL * kColChunk) {
            float x[VEC][kColChunk];
#pragma unroll
            for (int q = 0; q < kColChunk; ++q) {
                const int64_t i = i0 + (int64_t)q * kColRL;
                float fi = -INFINITY;
                if (i < r_hi) fi = __ldg(fb + i);
                if (fi != -INFINITY) {  // warp-uniform: a warp is one row lane
                    if constexpr (VEC == 4) {
                        const float4 c = ld_c4<T>(Cb + i * a.sCn + j0);
                        const float2 f2 = make_float2(fi, fi);
                        const float2 x01 = scaled_diff2(f2, make_float2(c.x, c.y), k);
                        const float2 x23 = scaled_diff2(f2, make_float2(c.z, c.w), k);
                        x[0][q] = x01.x;
                        x[1][q] = x01.y;
                        x[2][q] = x23.x;
                        x[3][q] = x23.y;
                    } else {
                        x[0][q] = (fi - ld_c1<T>(Cb + i * a.sCn + j0 * a.sCm)) * k;
                    }
                } else {
#pragma unroll
                    for (int v = 0; v < VEC; ++v) x[v][q] = -INFINITY;
                }
            }
            if constexpr (VEC == 4) {
                lse_fold_x2<kColChunk>(m[0], s[0], m[1], s[1], x[0], x[1]);
                lse_fold_x2<kColChunk>(m[2], s[2], m[3], s[3], x[2], x[3]);
            } else {
#pragma unroll
                for (int v = 0; v < VEC; ++v) lse_fold<kColChunk>(m[v], s[v], x[v]);
            }
        }
    }
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
        sh_m[rl][ct * VEC + v] = m[v];
        sh_s[rl][ct * VEC + v] = s[v];
    }
    col_tail<TJ>(a, b, tile, band, iter, check, &sh_m[0][0], &sh_s[0][0], sh_res, &sh_last);
}

}  // namespace sk
