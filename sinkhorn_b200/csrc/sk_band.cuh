// sk_band.cuh -- one pass over C producing weighted exp-sums along rows and
// columns at once.
//
// For every entry the kernel forms
//     t_ij = ((u_i + v_j) - C_ij) / eps + alpha_i + beta_j       (natural log)
//     p_ij = exp(t_ij)            or p_ij = P_ij (a materialised plan)
//     w_ij = p_ij * [gP_ij] * [C_ij] * scale
// (bracketed factors optional, missing vectors are 0, masked rows/columns give
// w = 0) and reduces
//     row0_i = sum_j w_ij wc_j   row1_i = sum_j w_ij
//     col0_j = sum_i w_ij wr_i   col1_j = sum_i w_ij
// optionally writing elem_ij = elem_scale * w_ij. Tiles are 32*VEC columns by
// a band of rows (the column-sweep layout, whole 512-byte row segments per
// warp): row sums are reduced across each warp and merged over tiles by the
// last CTA of a band, column sums are merged over bands by the last CTA of a
// tile (atomic tickets; no spin waits).
//
// Uses: the P-free JVP of jvp_kernel.py:11-110, the plan adjoint, the cost
// <P, C>, and the reverse sweeps of the backward.
#pragma once

#include "sk_common.cuh"

namespace sk {

constexpr int kBandRowsPerStep = 4;  // rows in flight per row lane

enum BandEpi : int {
    EPI_RAW = 0,  // row_out0/1 = row sums, col_out0/1 = column sums
    EPI_JVP = 1,  // out_f = mix(rho_a, wr, row0/max(row1,tiny)), same for g
};

struct BandArgs {
    const float* C;
    int64_t sCb, sCn, sCm;
    int64_t B, N, M;
    const float* P;        // dense plan (B,N,M) replacing exp(t), or nullptr
    const float* gP;       // dense multiplier (B,N,M), or nullptr
    const float* u;        // (B,N) or nullptr
    const float* alpha;    // (B,N) or nullptr
    const float* wr;       // (B,N) column-sum weights or nullptr (1)
    const float* v;        // (B,M) or nullptr
    const float* beta;     // (B,M) or nullptr
    const float* wc;       // (B,M) row-sum weights or nullptr (1)
    const uint8_t* mask_a; // (B,N) or nullptr
    const uint8_t* mask_b; // (B,M) or nullptr
    float inv_eps, scale;
    float khi, klo;        // log2(e)/eps as a float pair (PRECISE path)
    int precise;           // launch_band: the PRECISE instance of k_band
    int times_c;           // multiply w by C_ij
    float* elem_out;       // dense (B,N,M) or nullptr
    float elem_scale;
    int row_q, col_q;      // number of row / column quantities (0, 1 = sum1 only, 2)
    float* row_part;       // [2][B*N*ntiles]
    float* col_part;       // [2][B*nbands*M]
    unsigned* tick_row;    // [B*nbands]
    unsigned* tick_col;    // [B*ntiles]
    float* row_out0;
    float* row_out1;
    float* col_out0;
    float* col_out1;
    int epi;
    float rho_a, omr_a, rho_b, omr_b;
    int64_t ntiles, nbands, band_rows;
    const int* skip;       // device flag: the pass returns at once when nonzero (k_band only)
};

// PRECISE: p = exp((u + v) - C) / eps) through exp_scaled (a few ulp; alpha
// and beta must be absent); the default multiplies by 1/eps and takes
// ex2.approx of t * log2(e), up to |t| * 2^-23 further off. The implicit
// adjoint's CG amplifies plan rounding by ~1e3 and needs PRECISE; everything
// else is within tolerance either way.
template <int VEC, bool PRECISE = false>
__global__ void __launch_bounds__(kColThreads) k_band(BandArgs a) {
    constexpr int TJ = kColCT * VEC;
    __shared__ float sh0[kColRL][TJ];
    __shared__ float sh1[kColRL][TJ];
    __shared__ int sh_last_col, sh_last_row;

    if (a.skip != nullptr && *a.skip != 0) return;  // set by an earlier launch on the stream
    const int64_t cta = blockIdx.x;
    const int64_t tile = cta % a.ntiles;
    const int64_t t2 = cta / a.ntiles;
    const int64_t band = t2 % a.nbands;
    const int64_t b = t2 / a.nbands;
    const int ct = threadIdx.x % kColCT, rl = threadIdx.x / kColCT;
    const int64_t j0 = tile * TJ + (int64_t)ct * VEC;
    const int64_t r_lo = band * a.band_rows;
    const int64_t r_hi = r_lo + a.band_rows < a.N ? r_lo + a.band_rows : a.N;
    const bool colok = j0 < a.M;

    // per-column constants, loaded once
    float vj[VEC], bj[VEC], wcj[VEC];
    bool cvalid[VEC];
#pragma unroll
    for (int q = 0; q < VEC; ++q) {
        const int64_t j = j0 + q;
        const bool in = colok && j < a.M;
        const int64_t col = b * a.M + j;
        vj[q] = (in && a.v) ? a.v[col] : 0.f;
        bj[q] = (in && a.beta) ? a.beta[col] : 0.f;
        wcj[q] = (in && a.wc) ? a.wc[col] : 1.f;
        cvalid[q] = in && (a.mask_b == nullptr || a.mask_b[col] != 0);
    }
    float cs0[VEC], cs1[VEC];
#pragma unroll
    for (int q = 0; q < VEC; ++q) cs0[q] = cs1[q] = 0.f;

    const float* Cb = a.C + b * a.sCb;
    const bool needc = (a.P == nullptr) || a.times_c;
    for (int64_t i0 = r_lo + rl; i0 < r_hi; i0 += (int64_t)kColRL * kBandRowsPerStep) {
        float c[kBandRowsPerStep][VEC];
        float pl[kBandRowsPerStep][VEC];
        float gp[kBandRowsPerStep][VEC];
#pragma unroll
        for (int s = 0; s < kBandRowsPerStep; ++s) {
            const int64_t i = i0 + (int64_t)s * kColRL;
#pragma unroll
            for (int q = 0; q < VEC; ++q) c[s][q] = pl[s][q] = gp[s][q] = 0.f;
            if (i < r_hi && colok) {
                const int64_t e = (b * a.N + i) * a.M + j0;  // dense index
                if constexpr (VEC == 4) {
                    if (needc) {
                        const float4 cc = ld_stream4(Cb + i * a.sCn + j0);
                        c[s][0] = cc.x; c[s][1] = cc.y; c[s][2] = cc.z; c[s][3] = cc.w;
                    }
                    if (a.P) {
                        const float4 pp = ld_stream4(a.P + e);
                        pl[s][0] = pp.x; pl[s][1] = pp.y; pl[s][2] = pp.z; pl[s][3] = pp.w;
                    }
                    if (a.gP) {
                        const float4 gg = ld_stream4(a.gP + e);
                        gp[s][0] = gg.x; gp[s][1] = gg.y; gp[s][2] = gg.z; gp[s][3] = gg.w;
                    }
                } else {
                    if (needc) c[s][0] = ld_stream1(Cb + i * a.sCn + j0 * a.sCm);
                    if (a.P) pl[s][0] = ld_stream1(a.P + e);
                    if (a.gP) gp[s][0] = ld_stream1(a.gP + e);
                }
            }
        }
#pragma unroll
        for (int s = 0; s < kBandRowsPerStep; ++s) {
            const int64_t i = i0 + (int64_t)s * kColRL;
            if (i >= r_hi) break;  // warp-uniform
            const int64_t row = b * a.N + i;
            const bool rvalid = a.mask_a == nullptr || a.mask_a[row] != 0;
            const float ui = a.u ? a.u[row] : 0.f;
            const float ai = a.alpha ? a.alpha[row] : 0.f;
            const float wri = a.wr ? a.wr[row] : 1.f;
            float w[VEC];
            float r0 = 0.f, r1 = 0.f;
#pragma unroll
            for (int q = 0; q < VEC; ++q) {
                float p;
                if (a.P) {
                    p = pl[s][q];
                } else {
                    if constexpr (PRECISE) {
                        p = exp_scaled((ui + vj[q]) - c[s][q], a.khi, a.klo);
                    } else {
                        const float t = ((ui + vj[q]) - c[s][q]) * a.inv_eps + (ai + bj[q]);
                        p = ex2(t * kLog2e);
                    }
                }
                float x = p * a.scale;
                if (a.gP) x *= gp[s][q];
                if (a.times_c) x *= c[s][q];
                w[q] = (rvalid && cvalid[q]) ? x : 0.f;
                r0 += w[q] * wcj[q];
                r1 += w[q];
                cs0[q] += w[q] * wri;
                cs1[q] += w[q];
            }
            if (a.elem_out && colok) {
                float* dst = a.elem_out + row * a.M + j0;
                if constexpr (VEC == 4) {
                    *reinterpret_cast<float4*>(dst) =
                        make_float4(a.elem_scale * w[0], a.elem_scale * w[1],
                                    a.elem_scale * w[2], a.elem_scale * w[3]);
                } else {
                    dst[0] = a.elem_scale * w[0];
                }
            }
            if (a.row_q > 0) {
                if (a.row_q > 1) r0 = warp_sum(r0);
                r1 = warp_sum(r1);
                if (ct == 0) {
                    const int64_t pidx = row * a.ntiles + tile;
                    if (a.row_q > 1) a.row_part[pidx] = r0;
                    a.row_part[(int64_t)a.B * a.N * a.ntiles + pidx] = r1;
                }
            }
        }
    }

    // ---- column partials of this band ----------------------------------
    if (a.col_q > 0) {
#pragma unroll
        for (int q = 0; q < VEC; ++q) {
            sh0[rl][ct * VEC + q] = cs0[q];
            sh1[rl][ct * VEC + q] = cs1[q];
        }
        __syncthreads();
        for (int cc = threadIdx.x; cc < TJ; cc += kColThreads) {
            const int64_t j = tile * TJ + cc;
            if (j >= a.M) continue;
            float s0 = 0.f, s1 = 0.f;
#pragma unroll
            for (int q = 0; q < kColRL; ++q) {
                s0 += sh0[q][cc];
                s1 += sh1[q][cc];
            }
            const int64_t pidx = (b * a.nbands + band) * a.M + j;
            a.col_part[pidx] = s0;
            a.col_part[(int64_t)a.B * a.nbands * a.M + pidx] = s1;
        }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        sh_last_col = 0;
        sh_last_row = 0;
        if (a.col_q > 0)
            sh_last_col = atomicAdd(&a.tick_col[b * a.ntiles + tile], 1u) ==
                          (unsigned)(a.nbands - 1);
        if (a.row_q > 0)
            sh_last_row = atomicAdd(&a.tick_row[b * a.nbands + band], 1u) ==
                          (unsigned)(a.ntiles - 1);
    }
    __syncthreads();
    if (sh_last_col) {
        __threadfence();
        for (int cc = threadIdx.x; cc < TJ; cc += kColThreads) {
            const int64_t j = tile * TJ + cc;
            if (j >= a.M) continue;
            float s0 = 0.f, s1 = 0.f;
            for (int64_t q = 0; q < a.nbands; ++q) {
                const int64_t pidx = (b * a.nbands + q) * a.M + j;
                s0 += __ldcg(a.col_part + pidx);
                s1 += __ldcg(a.col_part + (int64_t)a.B * a.nbands * a.M + pidx);
            }
            const int64_t col = b * a.M + j;
            if (a.epi == EPI_JVP) {
                float r = s0 / fmaxf(s1, kTiny);
                if (a.rho_b != 0.f) r = a.rho_b * a.wc[col] + a.omr_b * r;
                a.col_out0[col] = r;
            } else {
                if (a.col_out0) a.col_out0[col] = s0;
                if (a.col_out1) a.col_out1[col] = s1;
            }
        }
        if (threadIdx.x == 0) a.tick_col[b * a.ntiles + tile] = 0u;
    }
    if (sh_last_row) {
        __threadfence();
        for (int64_t i = r_lo + threadIdx.x; i < r_hi; i += kColThreads) {
            const int64_t row = b * a.N + i;
            float s0 = 0.f, s1 = 0.f;
            for (int64_t q = 0; q < a.ntiles; ++q) {
                const int64_t pidx = row * a.ntiles + q;
                if (a.row_q > 1) s0 += __ldcg(a.row_part + pidx);
                s1 += __ldcg(a.row_part + (int64_t)a.B * a.N * a.ntiles + pidx);
            }
            if (a.epi == EPI_JVP) {
                float r = s0 / fmaxf(s1, kTiny);
                if (a.rho_a != 0.f) r = a.rho_a * a.wr[row] + a.omr_a * r;
                a.row_out0[row] = r;
            } else {
                if (a.row_out0) a.row_out0[row] = s0;
                if (a.row_out1) a.row_out1[row] = s1;
            }
        }
        if (threadIdx.x == 0) a.tick_row[b * a.nbands + band] = 0u;
    }
}

// ---------------------------------------------------------------------------
// Lean forms of the two single-direction passes of the backward (row sums
// R_i = sum_j wc_j w_ij with w_ij = exp((u_i - C_ij)/eps + beta_j), column
// sums S_j = sum_i wr_i w_ij with w_ij = exp((v_j - C_ij)/eps + alpha_i);
// arguments are log-plan entries, so no running max). launch_band routes an
// argument set of exactly that shape here (float4 layout); results are those
// of k_band up to summation order.

// Row sums in the row layout: persistent CTAs, each warp streaming RW rows of
// one item at once; one warp reduction per row (not one per 128-column tile).
template <int RW, int U>
__global__ void __launch_bounds__(kRowThreads) k_band_rows(BandArgs a) {
    constexpr int NW = kRowThreads / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float k2 = a.inv_eps * kLog2e;
    const int64_t nv = a.M >> 2;
    const int64_t gpi = (a.N + RW - 1) / RW;
    const int64_t ngroups = a.B * gpi;
    const int64_t wstride = (int64_t)gridDim.x * NW;
    for (int64_t grp = (int64_t)blockIdx.x * NW + warp; grp < ngroups; grp += wstride) {
        const int64_t b = grp / gpi;
        const int64_t i0 = (grp - b * gpi) * RW;
        const float* beta = a.beta ? a.beta + b * a.M : nullptr;
        const float* wc = a.wc ? a.wc + b * a.M : nullptr;
        const uint8_t* mb = a.mask_b ? a.mask_b + b * a.M : nullptr;
        const float* Crow[RW];
        bool rv[RW];
        float ur[RW], r0[RW], r1[RW];
#pragma unroll
        for (int r = 0; r < RW; ++r) {
            const int64_t i = i0 + r;
            const int64_t row = b * a.N + i;
            rv[r] = i < a.N && (a.mask_a == nullptr || a.mask_a[row] != 0);
            ur[r] = (rv[r] && a.u) ? a.u[row] : 0.f;
            Crow[r] = a.C + b * a.sCb + (rv[r] ? i : 0) * a.sCn;
            r0[r] = r1[r] = 0.f;
        }
        for (int64_t v = lane; v < nv; v += (int64_t)U * 32) {
            float bt[U][4], wcv[U][4];
            bool cv[U][4];
            float4 c[RW][U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int64_t vv = v + 32 * u;
                const bool in = vv < nv;
                const float4 b4 = (in && beta) ? ld_vec4(beta + 4 * vv) : make_float4(0.f, 0.f, 0.f, 0.f);
                const float4 w4 = (in && wc) ? ld_vec4(wc + 4 * vv) : make_float4(1.f, 1.f, 1.f, 1.f);
                uchar4 m4 = make_uchar4(1, 1, 1, 1);
                if (in && mb) m4 = *reinterpret_cast<const uchar4*>(mb + 4 * vv);
                bt[u][0] = b4.x * kLog2e; bt[u][1] = b4.y * kLog2e;
                bt[u][2] = b4.z * kLog2e; bt[u][3] = b4.w * kLog2e;
                wcv[u][0] = w4.x; wcv[u][1] = w4.y; wcv[u][2] = w4.z; wcv[u][3] = w4.w;
                cv[u][0] = in && m4.x; cv[u][1] = in && m4.y;
                cv[u][2] = in && m4.z; cv[u][3] = in && m4.w;
#pragma unroll
                for (int r = 0; r < RW; ++r)
                    c[r][u] = (in && rv[r]) ? ld_stream4(Crow[r] + 4 * vv)
                                            : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int r = 0; r < RW; ++r) {
                if (!rv[r]) continue;
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const float cc[4] = {c[r][u].x, c[r][u].y, c[r][u].z, c[r][u].w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float w = cv[u][e] ? ex2(fmaf(ur[r] - cc[e], k2, bt[u][e])) : 0.f;
                        r0[r] = fmaf(w, wcv[u][e], r0[r]);
                        r1[r] += w;
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < RW; ++r) {
            r0[r] = warp_sum(r0[r]);
            r1[r] = warp_sum(r1[r]);
        }
        if (lane == 0) {
#pragma unroll
            for (int r = 0; r < RW; ++r) {
                if (i0 + r >= a.N) break;
                const int64_t row = b * a.N + i0 + r;
                if (a.row_out0) a.row_out0[row] = r0[r];
                if (a.row_out1) a.row_out1[row] = r1[r];
            }
        }
    }
}

// Column sums in the column layout of k_band, without its row-sum and
// optional-factor work; each step's per-row constants are loaded with its C.
template <int VEC>
__global__ void __launch_bounds__(kColThreads) k_band_cols(BandArgs a) {
    constexpr int TJ = kColCT * VEC;
    constexpr int S = kBandRowsPerStep;
    __shared__ float sh0[kColRL][TJ];
    __shared__ float sh1[kColRL][TJ];
    __shared__ int sh_last;
    const int64_t cta = blockIdx.x;
    const int64_t tile = cta % a.ntiles;
    const int64_t t2 = cta / a.ntiles;
    const int64_t band = t2 % a.nbands;
    const int64_t b = t2 / a.nbands;
    const int ct = threadIdx.x % kColCT, rl = threadIdx.x / kColCT;
    const int64_t j0 = tile * TJ + (int64_t)ct * VEC;
    const int64_t r_lo = band * a.band_rows;
    const int64_t r_hi = r_lo + a.band_rows < a.N ? r_lo + a.band_rows : a.N;
    const bool colok = j0 < a.M;
    const float k2 = a.inv_eps * kLog2e;
    float vj[VEC], cs0[VEC], cs1[VEC];
    bool cvalid[VEC];
#pragma unroll
    for (int q = 0; q < VEC; ++q) {
        const int64_t col = b * a.M + j0 + q;
        const bool in = colok && j0 + q < a.M;
        vj[q] = (in && a.v) ? a.v[col] : 0.f;
        cvalid[q] = in && (a.mask_b == nullptr || a.mask_b[col] != 0);
        cs0[q] = cs1[q] = 0.f;
    }
    const float* Cb = a.C + b * a.sCb;
    for (int64_t i0 = r_lo + rl; i0 < r_hi; i0 += (int64_t)kColRL * S) {
        float c[S][VEC], ar[S], wr[S];
#pragma unroll
        for (int s = 0; s < S; ++s) {
            const int64_t i = i0 + (int64_t)s * kColRL;
#pragma unroll
            for (int q = 0; q < VEC; ++q) c[s][q] = 0.f;
            ar[s] = -INFINITY;  // rows past the band or masked contribute 0
            wr[s] = 0.f;
            if (i < r_hi) {
                const int64_t row = b * a.N + i;
                if (a.mask_a == nullptr || a.mask_a[row] != 0) {
                    ar[s] = a.alpha ? a.alpha[row] * kLog2e : 0.f;
                    wr[s] = a.wr ? a.wr[row] : 1.f;
                }
                if (colok) {
                    if constexpr (VEC == 4) {
                        const float4 cc = ld_stream4(Cb + i * a.sCn + j0);
                        c[s][0] = cc.x; c[s][1] = cc.y; c[s][2] = cc.z; c[s][3] = cc.w;
                    } else {
                        c[s][0] = ld_stream1(Cb + i * a.sCn + j0 * a.sCm);
                    }
                }
            }
        }
#pragma unroll
        for (int s = 0; s < S; ++s) {
#pragma unroll
            for (int q = 0; q < VEC; ++q) {
                const float w = ex2(fmaf(vj[q] - c[s][q], k2, ar[s]));
                cs0[q] = fmaf(w, wr[s], cs0[q]);
                cs1[q] += w;
            }
        }
    }
#pragma unroll
    for (int q = 0; q < VEC; ++q) {
        if (!cvalid[q]) cs0[q] = cs1[q] = 0.f;
        sh0[rl][ct * VEC + q] = cs0[q];
        sh1[rl][ct * VEC + q] = cs1[q];
    }
    __syncthreads();
    for (int cc = threadIdx.x; cc < TJ; cc += kColThreads) {
        const int64_t j = tile * TJ + cc;
        if (j >= a.M) continue;
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int q = 0; q < kColRL; ++q) {
            s0 += sh0[q][cc];
            s1 += sh1[q][cc];
        }
        const int64_t pidx = (b * a.nbands + band) * a.M + j;
        a.col_part[pidx] = s0;
        a.col_part[(int64_t)a.B * a.nbands * a.M + pidx] = s1;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0)
        sh_last = atomicAdd(&a.tick_col[b * a.ntiles + tile], 1u) == (unsigned)(a.nbands - 1);
    __syncthreads();
    if (!sh_last) return;
    __threadfence();
    for (int cc = threadIdx.x; cc < TJ; cc += kColThreads) {
        const int64_t j = tile * TJ + cc;
        if (j >= a.M) continue;
        float s0 = 0.f, s1 = 0.f;
        for (int64_t q = 0; q < a.nbands; ++q) {
            const int64_t pidx = (b * a.nbands + q) * a.M + j;
            s0 += __ldcg(a.col_part + pidx);
            s1 += __ldcg(a.col_part + (int64_t)a.B * a.nbands * a.M + pidx);
        }
        const int64_t col = b * a.M + j;
        if (a.col_out0) a.col_out0[col] = s0;
        if (a.col_out1) a.col_out1[col] = s1;
    }
    if (threadIdx.x == 0) a.tick_col[b * a.ntiles + tile] = 0u;
}

// Host side (sk_plan.cu): workspace bytes of one band pass and its launch.
size_t band_workspace_bytes(int64_t B, int64_t N, int64_t M);
// Fills the plan fields of `a` (tiles, bands, partial buffers, tickets) from
// the workspace, zeroes the tickets and launches. `vec4` selects the float4
// path (C, P and gP contiguous and 16-byte aligned, M % 4 == 0).
int launch_band(BandArgs a, bool vec4, void* ws, cudaStream_t s);

// The persistent plan pass (sk_implicit.cu) for plain row / column sums of
// the P-free plan: row0 = sum_j p x_j, col0 = sum_i p y_i (x, y nullptr = 1)
// and, with `dual`, row1 = sum_j p, col1 = sum_i p, each finished (any output
// may be nullptr); `times_c` weighs each term by C as well (row sums only).
// Returns kPlanSumsUnsuited, queueing nothing, when the
// operands do not fit it (strided C, unaligned rows or vectors); the caller
// then runs its band pass. `ws` holds plan_sums_bytes(B, N, M, dual).
constexpr int kPlanSumsUnsuited = -1;
size_t plan_sums_bytes(int64_t B, int64_t N, int64_t M, bool dual);
int plan_sums(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb, int64_t sCn,
              int64_t sCm, const float* f, const float* g, double epsilon,
              const uint8_t* mask_a, const uint8_t* mask_b, const float* x, const float* y,
              bool dual, float* row0, float* row1, float* col0, float* col1, void* ws,
              cudaStream_t s, bool times_c = false);

// The float4 path needs C contiguous along columns and 16-byte aligned rows.
inline bool vec4_ok(const float* C, int64_t B, int64_t M, int64_t sCb, int64_t sCn,
                    int64_t sCm) {
    return ((uintptr_t)C % 16 == 0) && sCm == 1 && M % 4 == 0 && sCn % 4 == 0 &&
           (B == 1 || sCb % 4 == 0);
}

inline bool dense_ok(const float* X, int64_t M) {
    return X == nullptr || (((uintptr_t)X % 16 == 0) && M % 4 == 0);
}

inline BandArgs band_base(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                          int64_t sCn, int64_t sCm, double eps) {
    BandArgs a{};
    a.C = C;
    a.sCb = sCb;
    a.sCn = sCn;
    a.sCm = sCm;
    a.B = B;
    a.N = N;
    a.M = M;
    a.inv_eps = (float)(1.0 / eps);
    {
        const double k = 1.4426950408889634 / eps;
        a.khi = (float)k;
        a.klo = (float)(k - (double)a.khi);
    }
    a.scale = 1.f;
    a.elem_scale = 1.f;
    a.epi = EPI_RAW;
    return a;
}

}  // namespace sk
