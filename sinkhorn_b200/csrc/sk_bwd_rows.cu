// sk_bwd_rows.cu -- one reverse step of the backward with a single read of C,
// for rows that fit one CTA's shared memory (512 <= M <= 2048).
//
// Reverse step k of the backward (sk_backward.cu) is, per row i and column j,
//   R_i   = sum_j gf_j exp((f^k_i - C_ij)/eps - lse_c^k_j)        (row pass)
//   ff_i  = (1 - rho_a) mask(Fb_i - R_i), Fb_i = rho_a mask(Fb_i - R_i)
//   S_j   = sum_i ff_i exp((g^{k-1}_j - C_ij)/eps - lse_r^k_i)    (column pass)
// (the adjoints of the f- and g-updates of src/sinkhorn/autograd.py:61-131,
// written out by hand). ff_i needs only row i's R_i, so the column pass can
// fold row i while it is still staged: C is read once per reverse step
// instead of twice. The terms are probabilities of a normalised plan (at
// most 1), so plain sums stay in range with no reference tracking.
//
// A CTA owns a chunk of consecutive rows of one batch item, the whole row
// width, in the role layout of sk_rows_stage.cuh:
//   * producer (warp 16): one cp.async.bulk per row, R = SR TPC rows per stage
//     (SR = 8 rows per thread) into a 3-stage ring;
//   * 16 consumer warps: thread t owns the float4 column group t % G for the SR
//     rows of row set t / G; it sums its rows' weighted terms against the
//     stage's f (posted two stages ahead), adds them over the warp and posts
//     the warp's sums, then folds the PREVIOUS stage's tile (read again from
//     the ring, which releases it after the fold) into its 4 column sums with
//     that stage's ff and lse_r;
//   * finisher (warp 17; lane r owns row r of every stage): adds the warps'
//     sums into R_i, applies the row adjoint step (mask, guard, rho split,
//     dlog_a) and posts ff_i and -lse_r_i for the fold.
// At the end each chunk writes its column sums; k_bwd_vec merges the chunks
// in a fixed order and takes the column adjoint step of step k - 1.
#include <algorithm>
#include <cmath>

#include "sk_internal.h"
#include "sk_rows_stage.cuh"
#include "sk_solve.cuh"

namespace sk {

struct BwdRowsArgs {
    const float* C;
    int64_t sCb, sCn;
    int64_t B, N, M;
    const float* fk;        // (B,N) f^k: potentials of the row pass
    const float* gprev;     // (B,M) g^{k-1}: potentials of the column pass
    const float* gf;        // (B,M) gf^k: column weights of the row pass
    const float* bc;        // (B,M) -lse_c^k, natural log (-inf: empty column)
    const float* lr;        // (B,N) lse_r^k, natural log (-inf: empty row)
    const uint8_t* mask_a;  // full mode: rows without terms and without adjoint, else nullptr
    const uint8_t* mask_b;  // full mode: columns without terms, else nullptr
    float* Fb;              // (B,N) adjoint of f, in place
    float* ff;              // (B,N) ff^k out
    float* ar;              // (B,N) -lse_r^k out (-inf: empty row)
    float* dlog_a;          // (B,N) accumulated, or nullptr
    float* parts;           // (chunks, pstride): each chunk's column sums S
    int64_t pstride;
    int64_t chunks, rows_per_chunk;
    float k2;               // log2(e) / eps
    float eps, rho, omr;
    int full;               // a guarded (empty) row passes no gradient
    int col_pass;           // 0: the last reverse step (no column sums)
    Status* st;             // error word of a wait that gave up
};

// Shared memory after the ring. Per-stage records alternate between two slots
// (stage t uses slot t & 1), rewritten for stage t + 2 only after every
// reader of stage t has passed the barrier that orders it.
struct BrTail {
    float2 fk[2][kRfMaxRows];         // (f, f): f^k of the stage's rows
    float2 ffar[2][kRfMaxRows];       // (ff, -lse_r log2(e)): the fold's row factors
    float wsum[2][kRfWarps][8];       // warps' row sums (SR per warp)
    uint64_t full[kRfStages];         // producer -> consumers: a stage landed
    uint64_t empty[kRfStages];        // consumer warps -> producer: a stage is folded
    uint64_t sums[2];                 // consumer warps -> finisher: row sums posted
    uint64_t fdone[2];                // finisher -> consumers: the stage's factors posted
    uint64_t rready;                  // finisher -> consumers: the first f posted
    int abort;
};

// rows of 2048 < M <= 4096 (V = 2: a thread owns two float4 groups of each
// row) stage 4 rows at a time in 3 stages: 48 M bytes of ring
constexpr int kBrMaxM = 4096;
static size_t br_smem_bytes(int64_t M) {
    return (M > kRfMaxM ? (size_t)3 * 4 * M * sizeof(float) : rf_ring_bytes(M)) + sizeof(BrTail);
}

template <int TPC, int V>
__global__ void __launch_bounds__(kRfThreads, 1) k_bwd_rows(BwdRowsArgs a) {
    static_assert(V == 1 || TPC == 1, "two column groups per thread only for the longest rows");
    constexpr int SR = V == 2 ? 4 : rf_set_rows<TPC>();  // rows per thread per stage
    constexpr int ST = V == 2 ? 3 : rf_stages<TPC>();    // stages
    constexpr int R = SR * TPC;                // rows per stage
    constexpr int G = kRfConsumers / TPC;      // column groups per row set
    constexpr int WPS = kRfWarps / TPC;        // warps per row set
    pdl_wait();
    pdl_trigger();
    extern __shared__ __align__(128) unsigned char br_smem[];
    const int64_t M = a.M;
    float* ring = reinterpret_cast<float*>(br_smem);  // [stages][R][M]
    BrTail& T = *reinterpret_cast<BrTail*>(ring + (size_t)ST * R * M);
    Status* st = a.st;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const int64_t b = blockIdx.x / a.chunks;
    const int64_t chunk = blockIdx.x % a.chunks;
    const int64_t r0 = chunk * a.rows_per_chunk;
    const int64_t r1 = std::max(r0, std::min<int64_t>(a.N, r0 + a.rows_per_chunk));
    const int64_t nstages = (r1 - r0 + R - 1) / R;

    if (threadIdx.x == 0) {
        for (int q = 0; q < ST; ++q) {
            mbar_init(&T.full[q], 1);
            mbar_init(&T.empty[q], kRfWarps);
        }
        for (int q = 0; q < 2; ++q) {
            mbar_init(&T.sums[q], kRfWarps);
            mbar_init(&T.fdone[q], 1);
        }
        mbar_init(&T.rready, 1);
        T.abort = 0;
        mbar_init_fence();
    }
    __syncthreads();
    volatile int* ab = &T.abort;
    const float k2 = a.k2;

    if (warp == kRfProducer) {
        // ---- producer: whole rows (M floats, 16-byte aligned) -------------
        const uint32_t bytes = (uint32_t)(sizeof(float) * M);
        const float* Cb = a.C + b * a.sCb;
        const int stage_floats = R * (int)M;  // ring offsets fit 32 bits
        float* dst0 = ring + lane * (int)M;
        int q = 0;
        uint32_t ph = 0u;
        int64_t t = 0;
        for (; t < nstages; ++t) {
            if (t >= ST &&
                !__all_sync(0xffffffffu, rf_wait(&T.empty[q], ph ^ 1u, ab)))
                break;
            const int64_t i = r0 + t * R + lane;
            const bool live = lane < R && i < r1;
            const unsigned n = __popc(__ballot_sync(0xffffffffu, live));
            if (lane == 0) mbar_expect_tx(&T.full[q], n * bytes);
            __syncwarp();
            if (live) bulk_g2s(dst0 + q * stage_floats, Cb + i * a.sCn, bytes, &T.full[q]);
            if (++q == ST) {
                q = 0;
                ph ^= 1u;
            }
        }
        if (t < nstages && lane == 0) rf_abort(ab, st);
        // every copy issued lands before the CTA can leave (bounded)
        const int64_t first = t > ST ? t - ST : 0;
        for (int64_t u = first; u < t; ++u)
            if (!mbar_wait(&T.full[u % ST], (uint32_t)(u / ST) & 1u) && lane == 0)
                rf_abort(ab, st);
        return;
    }

    if (warp == kRfFinisher) {
        // ---- finisher: lane r < R owns row r of every stage ---------------
        // a row's inputs, loaded three stages ahead (flags: 1 in the chunk,
        // 2 masked)
        struct RowIn {
            float fk, Fb, lr, dl;
            int fl;
        };
        auto row_load = [&](int64_t t) {
            RowIn v{0.f, 0.f, -INFINITY, 0.f, 0};
            const int64_t i = r0 + t * R + lane;
            if (lane < R && t < nstages && i < r1) {
                const int64_t row = b * a.N + i;
                v.fk = a.fk[row];
                v.Fb = a.Fb[row];
                v.lr = a.lr[row];
                if (a.dlog_a) v.dl = a.dlog_a[row];
                v.fl = 1 | ((a.mask_a && !a.mask_a[row]) ? 2 : 0);
            }
            return v;
        };
        RowIn v0 = row_load(0), v1 = row_load(1), v2 = row_load(2);
        if (lane < R) {
            T.fk[0][lane] = make_float2(v0.fk, v0.fk);
            T.fk[1][lane] = make_float2(v1.fk, v1.fk);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&T.rready);
        for (int64_t t = 0; t < nstages; ++t) {
            const int sl = (int)(t & 1);
            if (!__all_sync(0xffffffffu, rf_wait(&T.sums[sl], (uint32_t)(t >> 1) & 1u, ab))) {
                if (lane == 0) rf_abort(ab, st);
                break;
            }
            if (lane < R) {
                float2 fa = make_float2(0.f, -INFINITY);  // past the chunk: no term
                if (v0.fl & 1) {
                    const int rset = lane / SR, k = lane % SR;
                    float Rs = 0.f;
#pragma unroll
                    for (int w = 0; w < WPS; ++w) Rs += T.wsum[sl][rset * WPS + w][k];
                    const int64_t row = b * a.N + r0 + t * R + lane;
                    const bool masked = (v0.fl & 2) != 0;
                    const float bar = masked ? 0.f : v0.Fb - Rs;
                    const bool empty = v0.lr == -INFINITY;
                    const float ffv = (a.full && empty) ? 0.f : a.omr * bar;
                    const float arv = empty ? -INFINITY : -v0.lr;
                    a.Fb[row] = a.rho * bar;
                    a.ff[row] = ffv;
                    a.ar[row] = arv;
                    if (a.dlog_a) a.dlog_a[row] = v0.dl + a.eps * (a.omr * bar);
                    fa = make_float2(ffv, masked ? -INFINITY : arv * kLog2e);
                }
                T.ffar[sl][lane] = fa;
                // f of stage t + 2 (this slot's readers are done with stage t)
                T.fk[sl][lane] = make_float2(v2.fk, v2.fk);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&T.fdone[sl]);
            v0 = v1;
            v1 = v2;
            v2 = row_load(t + 3);
        }
        return;
    }

    // ---- consumers ---------------------------------------------------------
    // thread tc owns the float4 groups u + G v (v < V) of its row set's rows
    const float2 kk = make_float2(k2, k2), neg1 = make_float2(-1.f, -1.f);
    const int tc = threadIdx.x;
    const int rs = tc / G;                 // row set: rows SR rs .. SR rs + SR - 1
    const int u = tc % G;
    int64_t jc[V];
    bool cols[V];
    float2 gf2[V][2], bc2[V][2], gp2[V][2];
    bool cv[V][4];
#pragma unroll
    for (int v = 0; v < V; ++v) {
        jc[v] = 4 * (int64_t)(u + G * v);
        cols[v] = jc[v] < M;
        float gfv[4] = {0.f, 0.f, 0.f, 0.f}, bcl[4], gpv[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            bcl[e] = -INFINITY;
            cv[v][e] = false;
        }
        if (cols[v]) {
            const int64_t o = b * M + jc[v];
            const float4 w4 = *reinterpret_cast<const float4*>(a.gf + o);
            const float4 c4 = *reinterpret_cast<const float4*>(a.bc + o);
            const float4 p4 = *reinterpret_cast<const float4*>(a.gprev + o);
            const float wv[4] = {w4.x, w4.y, w4.z, w4.w}, bv[4] = {c4.x, c4.y, c4.z, c4.w};
            const float pv[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                cv[v][e] = a.mask_b == nullptr || a.mask_b[o + e] != 0;
                gfv[e] = wv[e];
                bcl[e] = cv[v][e] ? bv[e] * kLog2e : -INFINITY;  // a masked column has no term
                gpv[e] = pv[e];
            }
        }
        gf2[v][0] = make_float2(gfv[0], gfv[1]);
        gf2[v][1] = make_float2(gfv[2], gfv[3]);
        bc2[v][0] = make_float2(bcl[0], bcl[1]);
        bc2[v][1] = make_float2(bcl[2], bcl[3]);
        gp2[v][0] = make_float2(gpv[0], gpv[1]);
        gp2[v][1] = make_float2(gpv[2], gpv[3]);
    }
    float2 S[V][2];
#pragma unroll
    for (int v = 0; v < V; ++v) S[v][0] = S[v][1] = make_float2(0.f, 0.f);
    if (!__all_sync(0xffffffffu, rf_wait(&T.rready, 0u, ab)) && lane == 0) rf_abort(ab, st);
    const int stage_floats = R * (int)M;
    const float* tile0 = ring + SR * rs * (int)M + 4 * u;  // group v at + 4 G v
    int q = 0, qp = 0;
    uint32_t ph = 0u;
#pragma unroll 2
    for (int64_t t = 0; t <= nstages; ++t) {
        float4 cc[SR][V];
        if (t < nstages) {
            // ---- this stage's tile (the stage stays until its fold)
            if (!__all_sync(0xffffffffu, rf_wait(&T.full[q], ph, ab)) && lane == 0)
                rf_abort(ab, st);
            const bool bad = *ab != 0;
            const float* tile = tile0 + q * stage_floats;
#pragma unroll
            for (int k = 0; k < SR; ++k)
#pragma unroll
                for (int v = 0; v < V; ++v)
                    cc[k][v] = (cols[v] && !bad)
                                   ? *reinterpret_cast<const float4*>(tile + k * (int)M + 4 * G * v)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
            qp = q;
            if (++q == ST) {
                q = 0;
                ph ^= 1u;
            }
            // ---- row sums: gf_j 2^((f - c) k2 + bc_j) over this thread's columns
            const int sl = (int)(t & 1);
            float ps[SR];
#pragma unroll
            for (int k = 0; k < SR; ++k) {
                const float2 f2 = T.fk[sl][SR * rs + k];
                float2 p = make_float2(0.f, 0.f);
#pragma unroll
                for (int v = 0; v < V; ++v) {
                    const float2 x01 = __ffma2_rn(
                        __ffma2_rn(make_float2(cc[k][v].x, cc[k][v].y), neg1, f2), kk, bc2[v][0]);
                    const float2 x23 = __ffma2_rn(
                        __ffma2_rn(make_float2(cc[k][v].z, cc[k][v].w), neg1, f2), kk, bc2[v][1]);
                    const float2 pv = __ffma2_rn(make_float2(ex2(x23.x), ex2(x23.y)), gf2[v][1],
                                                 __fmul2_rn(make_float2(ex2(x01.x), ex2(x01.y)),
                                                            gf2[v][0]));
                    if (cols[v]) p = __fadd2_rn(p, pv);
                }
                ps[k] = p.x + p.y;
            }
            float s2;
            if constexpr (SR == 8) {
                s2 = rf_warp_rows8(ps, lane);
                if ((lane & 3) == 0) T.wsum[sl][warp][lane >> 2] = s2;
            } else {
                s2 = rf_warp_rows4(ps, lane);
                if ((lane & 7) == 0) T.wsum[sl][warp][lane >> 3] = s2;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&T.sums[sl]);
        }
        if (t > 0) {
            // ---- the previous stage: its row factors are posted
            const int64_t s = t - 1;
            const int sl = (int)(s & 1);
            if (!__all_sync(0xffffffffu, rf_wait(&T.fdone[sl], (uint32_t)(s >> 1) & 1u, ab)) &&
                lane == 0)
                rf_abort(ab, st);
            // ---- column fold: ff_i 2^((g - c) k2 - lse_r_i log2(e)) of the
            // previous stage's slot, still in the ring and released after it
            const int qf = t < nstages ? (qp == 0 ? ST - 1 : qp - 1) : qp;
            if (a.col_pass && *ab == 0) {
                const float* tp = tile0 + qf * stage_floats;
#pragma unroll
                for (int k = 0; k < SR; ++k) {
                    const float2 fa = T.ffar[sl][SR * rs + k];
                    if (fa.y == -INFINITY) continue;  // masked, empty or past the chunk
                    const float2 ar2 = make_float2(fa.y, fa.y), ff2 = make_float2(fa.x, fa.x);
#pragma unroll
                    for (int v = 0; v < V; ++v) {
                        if (!cols[v]) continue;
                        const float4 cpk =
                            *reinterpret_cast<const float4*>(tp + k * (int)M + 4 * G * v);
                        const float2 x01 = __ffma2_rn(
                            __ffma2_rn(make_float2(cpk.x, cpk.y), neg1, gp2[v][0]), kk, ar2);
                        const float2 x23 = __ffma2_rn(
                            __ffma2_rn(make_float2(cpk.z, cpk.w), neg1, gp2[v][1]), kk, ar2);
                        S[v][0] = __ffma2_rn(make_float2(ex2(x01.x), ex2(x01.y)), ff2, S[v][0]);
                        S[v][1] = __ffma2_rn(make_float2(ex2(x23.x), ex2(x23.y)), ff2, S[v][1]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&T.empty[qf]);
        }
    }
    if (!a.col_pass) return;

    float cs[V][4];
#pragma unroll
    for (int v = 0; v < V; ++v) {
        cs[v][0] = S[v][0].x;
        cs[v][1] = S[v][0].y;
        cs[v][2] = S[v][1].x;
        cs[v][3] = S[v][1].y;
    }
    // the row sets' column sums add up (through the ring, now idle), then the
    // chunk's row of the partials
    if constexpr (TPC > 1) {
        rf_consumers_sync();  // every consumer is past its last stage
        float4* scratch = reinterpret_cast<float4*>(ring);  // [TPC][G]
        scratch[(size_t)rs * G + u] = make_float4(cs[0][0], cs[0][1], cs[0][2], cs[0][3]);
        rf_consumers_sync();
        if (rs == 0) {
            for (int r2 = 1; r2 < TPC; ++r2) {
                const float4 o = scratch[(size_t)r2 * G + tc];
                cs[0][0] += o.x;
                cs[0][1] += o.y;
                cs[0][2] += o.z;
                cs[0][3] += o.w;
            }
        }
    }
    if (rs == 0) {
#pragma unroll
        for (int v = 0; v < V; ++v) {
            if (!cols[v]) continue;
            float* dst = a.parts + chunk * a.pstride + b * M + jc[v];
            *reinterpret_cast<float4*>(dst) =
                make_float4(cv[v][0] ? cs[v][0] : 0.f, cv[v][1] ? cs[v][1] : 0.f,
                            cv[v][2] ? cs[v][2] : 0.f, cv[v][3] ? cs[v][3] : 0.f);
        }
    }
}

template <int TPC, int V>
static int launch_bwd_rows_t(const BwdRowsArgs& a, cudaStream_t s) {
    static thread_local int done[64] = {0};
    int dev = 0;
    SK_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || !done[dev]) {
        SK_CUDA(cudaFuncSetAttribute(k_bwd_rows<TPC, V>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)br_smem_bytes(V == 2 ? kBrMaxM : 2048 / TPC)));
        if (dev >= 0 && dev < 64) done[dev] = 1;
    }
    launch_pdl(k_bwd_rows<TPC, V>, dim3((unsigned)(a.B * a.chunks)), dim3(kRfThreads),
               br_smem_bytes(a.M), s, a);
    SK_LAUNCHED("k_bwd_rows launch");
    return SK_OK;
}

bool bwd_rows_shape(const SweepPlan& p, int64_t N, int64_t M) {
    return p.fused_ok && !p.bf16 && p.vec == 4 && M % 4 == 0 && M >= kRfMinM && M <= kBrMaxM &&
           N >= 1;
}

int64_t bwd_rows_chunks(int64_t B, int64_t N, int64_t M) {
    return std::max<int64_t>(1, std::min(rows_fused_chunks(B, N), fused_max_chunks(B, N, M)));
}

int launch_bwd_rows(const Problem& P, const BwdRowsStep& r, cudaStream_t s) {
    BwdRowsArgs a{};
    a.C = P.C;
    a.sCb = P.sCb;
    a.sCn = P.sCn;
    a.B = P.B;
    a.N = P.N;
    a.M = P.M;
    a.fk = r.fk;
    a.gprev = r.gprev;
    a.gf = r.gf;
    a.bc = r.bc;
    a.lr = r.lr;
    a.mask_a = r.mask_a;
    a.mask_b = r.mask_b;
    a.Fb = r.Fb;
    a.ff = r.ff;
    a.ar = r.ar;
    a.dlog_a = r.dlog_a;
    a.parts = r.parts;
    a.pstride = r.pstride;
    a.chunks = r.chunks;
    a.rows_per_chunk = (P.N + r.chunks - 1) / r.chunks;
    a.k2 = r.k2;
    a.eps = r.eps;
    a.rho = r.rho;
    a.omr = r.omr;
    a.full = r.full;
    a.col_pass = r.col_pass;
    a.st = (Status*)r.status;
    if (P.M > kRfMaxM) return launch_bwd_rows_t<1, 2>(a, s);
    switch (rf_tpc(P.M)) {
        case 4: return launch_bwd_rows_t<4, 1>(a, s);
        case 2: return launch_bwd_rows_t<2, 1>(a, s);
        default: return launch_bwd_rows_t<1, 1>(a, s);
    }
}

}  // namespace sk
