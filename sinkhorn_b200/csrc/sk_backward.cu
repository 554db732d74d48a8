// sk_backward.cu -- backward of the Sinkhorn solve (C ABI sk_backward).
//
// SinkhornFunction.backward (src/sinkhorn/autograd.py:61-131) re-runs K
// iterations under autograd and back-propagates <f, grad_f> + <g, grad_g>.
// Here the K iterations are re-run with the forward's kernels (the
// single-read step and its finish where the forward takes them, else the
// two sweeps), keeping only the vectors f^k, g^k and the row/column LSEs
// (O(K(N+M)) memory instead of autograd's O(K N M) tape). The reverse pass is written out by hand: with
//   pi_r^k = exp((g^{k-1}_j - C_ij)/eps - lse_r^k_i)
//   pi_c^k = exp((f^k_i     - C_ij)/eps - lse_c^k_j)
// and adjoints Fb (of f^k), Gb (of g^k), for k = K..1:
//   gf^k = (1-rho_b) Gb            ; Gprev = rho_b Gb ; dlog_b += eps gf^k
//   Fb  -= sum_j gf^k_j pi_c^k_ij                      (band pass, rows)
//   ff^k = (1-rho_a) Fb            ; Fb = rho_a Fb    ; dlog_a += eps ff^k
//   Gb   = Gprev - sum_i ff^k_i pi_r^k_ij               (band pass, columns)
// and finally, in one pass over C that writes dC once,
//   dC_ij = sum_k gf^k_j pi_c^k_ij + ff^k_i pi_r^k_ij.
// Full mode (a fresh masked solve from zeros, checked every iteration) zeroes
// adjoints at masked entries before each half-step, gives masked entries of
// C no gradient and blocks the gradient of a guarded (empty) softmin;
// truncated mode runs on raw C and masks only the final potentials.
#include <cmath>

#include "sk_band.cuh"
#include "sk_internal.h"
#include "sk_solve.cuh"

namespace sk {

struct BwdVecArgs {
    int64_t n;             // B*N (row step) or B*M (column step)
    const uint8_t* mask;   // mask applied to the adjoint in full mode, or nullptr
    const float* lse;      // LSE of this half-step (natural log)
    float* adj;            // Fb or Gb (in/out)
    const float* sub;      // row step: R (subtracted from Fb); col step: S or nullptr
    const float* prev;     // col step: Gprev of the previous reverse step (or nullptr)
    float* keep;           // col step: Gprev out (rho * adj)
    float* w_out;          // gf^k / ff^k
    float* off_out;        // -lse (or -inf for an empty half-step)
    float* dlog;           // dlog_a / dlog_b accumulators (or nullptr)
    float rho, omr, eps;
    int full;
    // col step after a single-read reverse step (sk_bwd_rows.cu): sub is the
    // sum of the chunks' column sums, taken in chunk order
    const float* parts;
    int nparts;
    int64_t pstride;
};

// Column step (first = the adjoint of g^K is already in adj):
//   Gb = (first ? adj : prev - sub); gbar = mask ? Gb : 0
//   gf = guard ? 0 : (1-rho) gbar; keep = rho gbar; dlog += eps (1-rho) gbar
// Row step: Fb -= sub; fbar = mask ? Fb : 0; ff = guard ? 0 : (1-rho) fbar;
//   Fb = rho fbar; dlog += eps (1-rho) fbar
__global__ void k_bwd_vec(BwdVecArgs a, int is_col, int first) {
    pdl_wait();
    pdl_trigger();
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= a.n) return;
    float x;
    if (is_col && !first && a.parts) {
        float S = 0.f;
        for (int c = 0; c < a.nparts; ++c) S += a.parts[(int64_t)c * a.pstride + t];
        x = a.prev[t] - S;
    } else if (is_col) {
        x = first ? a.adj[t] : a.prev[t] - a.sub[t];
    } else {
        x = a.adj[t] - a.sub[t];
    }
    const bool masked = a.full && a.mask && !a.mask[t];
    const float bar = masked ? 0.f : x;
    const float l = a.lse[t];
    const bool empty = (l == -INFINITY);
    const bool guarded = a.full && empty;
    a.w_out[t] = guarded ? 0.f : a.omr * bar;
    a.off_out[t] = empty ? -INFINITY : -l;
    if (a.dlog) a.dlog[t] += a.eps * (a.omr * bar);
    if (is_col) {
        a.keep[t] = a.rho * bar;
        a.adj[t] = x;
    } else {
        a.adj[t] = a.rho * bar;
    }
}

// Fb = mask_a ? grad_f : 0, Gb = mask_b ? grad_g : 0 (final masking).
__global__ void k_bwd_seed(const float* grad, const uint8_t* mask, float* adj, int64_t n) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n) return;
    adj[t] = (mask && !mask[t]) ? 0.f : (grad ? grad[t] : 0.f);
}

// ---------------------------------------------------------------------------
// dC_ij = sum_k gf^k_j exp((f^k_i - C_ij)/eps + bc^k_j)
//              + ff^k_i exp((g^{k-1}_j - C_ij)/eps + ar^k_i)
// One CTA covers 32*VEC columns x (8 row lanes x kDcRows rows); C is read
// once into registers and dC written once. The per-iteration vectors of the
// CTA's columns and rows are staged in shared memory kDcKChunk iterations at a
// time (the -lse offsets pre-scaled to log2 units), so the K loop runs with no
// global load.
// Both terms of an iteration share exp(-C_ij/eps): in log2 units, with
// t1 = (f_i - c) k2 + bc_j, the second exponent is t1 + Q_j - P_i where
// Q_j = g_j k2 - bc_j and P_i = f_i k2 - ar_i, so the iteration's term is
// 2^t1 (gf_j + V_i U_j) with U_j = 2^(Q_j - Qr) and V_i = ff_i 2^(Qr - P_i),
// Qr the largest finite Q_j of the CTA's columns: one exponential per
// element. The CTA takes that form for an iteration when Qr - min P_i <= 40
// over its rows (U <= 1, V <= |ff| 2^40, and a term lost to 2^t1 flushing is
// below 2^-86 |ff|); a column without terms (bc = -inf: its C is +inf on
// every valid row) or a masked one gets U = 0, a row without terms V = 0.
// Otherwise (a NaN among the factors, or a wider spread, as far from
// convergence) it takes both exponentials.
constexpr float kDcSpread = 40.f;
constexpr int kDcRows = 4;
constexpr int kDcKChunk = 16;

struct DcArgs {
    const float* C;
    int64_t sCb, sCn, sCm;
    int64_t B, N, M;
    int K;
    int64_t BN, BM;        // history strides
    const float* hf;       // f^k at hf + k*BN, k = 0..K
    const float* hg;       // g^k at hg + k*BM
    const float* ff;       // ff^k at ff + (k-1)*BN
    const float* ar;       // -lse_r^k at ar + (k-1)*BN
    const float* gf;       // gf^k at gf + (k-1)*BM
    const float* bc;       // -lse_c^k at bc + (k-1)*BM
    const uint8_t* mask_a; // full mode only
    const uint8_t* mask_b;
    float k2;              // log2(e) / eps
    float* dC;             // dense (B,N,M)
    int64_t ntiles, nrowblk;
};

template <int VEC>
__global__ void __launch_bounds__(kColThreads) k_bwd_dc(DcArgs a) {
    constexpr int TJ = kColCT * VEC;
    constexpr int RB = kColRL * kDcRows;  // rows per CTA
    __shared__ __align__(16) float s_gf[kDcKChunk][TJ];
    __shared__ __align__(16) float s_bc[kDcKChunk][TJ];  // log2 units
    __shared__ __align__(16) float s_hg[kDcKChunk][TJ];
    __shared__ float s_hf[kDcKChunk][RB];
    __shared__ float s_ff[kDcKChunk][RB];
    __shared__ float s_ar[kDcKChunk][RB];  // log2 units
    __shared__ __align__(16) float s_u[kDcKChunk][TJ];  // Q_j, then U_j
    __shared__ float s_v[kDcKChunk][RB];                // P_i, then V_i
    __shared__ float s_qr[kDcKChunk];
    __shared__ int s_one[kDcKChunk];                    // 1: one exponential per element
    const int64_t cta = blockIdx.x;
    const int64_t tile = cta % a.ntiles;
    const int64_t t2 = cta / a.ntiles;
    const int64_t rb = t2 % a.nrowblk;
    const int64_t b = t2 / a.nrowblk;
    const int ct = threadIdx.x % kColCT, rl = threadIdx.x / kColCT;
    const int64_t j0 = tile * TJ + (int64_t)ct * VEC;
    const bool colok = j0 < a.M;  // every thread stays for the staging barriers
    const float k2 = a.k2;

    float c[kDcRows][VEC], acc[kDcRows][VEC];
    bool rv[kDcRows];
    int64_t rows[kDcRows];
    bool cv[VEC];
#pragma unroll
    for (int q = 0; q < VEC; ++q)
        cv[q] = colok && (a.mask_b == nullptr || a.mask_b[b * a.M + j0 + q] != 0);
#pragma unroll
    for (int s = 0; s < kDcRows; ++s) {
        const int64_t i = rb * RB + rl + (int64_t)s * kColRL;
        rows[s] = i;
        rv[s] = i < a.N && (a.mask_a == nullptr || a.mask_a[b * a.N + i] != 0);
#pragma unroll
        for (int q = 0; q < VEC; ++q) {
            acc[s][q] = 0.f;
            c[s][q] = 0.f;
        }
        if (i < a.N && colok) {
            const float* src = a.C + b * a.sCb + i * a.sCn;
            if constexpr (VEC == 4) {
                const float4 cc = ld_stream4(src + j0);
                c[s][0] = cc.x; c[s][1] = cc.y; c[s][2] = cc.z; c[s][3] = cc.w;
            } else {
                c[s][0] = ld_stream1(src + j0 * a.sCm);
            }
        }
    }
    for (int kc = 1; kc <= a.K; kc += kDcKChunk) {
        const int nk = a.K - kc + 1 < kDcKChunk ? a.K - kc + 1 : kDcKChunk;
        __syncthreads();  // the previous chunk is consumed
        for (int e = threadIdx.x; e < nk * TJ; e += kColThreads) {
            const int kk = e / TJ, cc = e - kk * TJ;
            const int64_t j = tile * TJ + cc;
            float gfv = 0.f, bcv = -INFINITY, hgv = 0.f;
            if (j < a.M) {
                const int64_t off = (int64_t)(kc + kk - 1) * a.BM + b * a.M + j;
                gfv = __ldg(a.gf + off);
                bcv = __ldg(a.bc + off) * kLog2e;
                hgv = __ldg(a.hg + off);  // g^{k-1}
            }
            s_gf[kk][cc] = gfv;
            s_bc[kk][cc] = bcv;
            s_hg[kk][cc] = hgv;
        }
        for (int e = threadIdx.x; e < nk * RB; e += kColThreads) {
            const int kk = e / RB, rr = e - kk * RB;
            const int64_t i = rb * RB + rr;
            float hfv = 0.f, ffv = 0.f, arv = -INFINITY;
            if (i < a.N) {
                const int64_t r = b * a.N + i;
                hfv = __ldg(a.hf + (int64_t)(kc + kk) * a.BN + r);  // f^k
                ffv = __ldg(a.ff + (int64_t)(kc + kk - 1) * a.BN + r);
                arv = __ldg(a.ar + (int64_t)(kc + kk - 1) * a.BN + r) * kLog2e;
            }
            s_hf[kk][rr] = hfv;
            s_ff[kk][rr] = ffv;
            s_ar[kk][rr] = arv;
            // P_i (+inf: a row without terms, or past N)
            s_v[kk][rr] = arv == -INFINITY ? INFINITY : hfv * k2 - arv;
        }
        for (int e = threadIdx.x; e < nk * TJ; e += kColThreads) {
            const int kk = e / TJ, cc = e - kk * TJ;
            const int64_t j = tile * TJ + cc;
            const bool live = j < a.M && (a.mask_b == nullptr || a.mask_b[b * a.M + j] != 0);
            // Q_j (-inf: excluded, a column without terms, masked or past M)
            const float q = s_hg[kk][cc] * k2 - s_bc[kk][cc];
            s_u[kk][cc] = (live && q != INFINITY) ? q : -INFINITY;
        }
        __syncthreads();
        {
            const int w = threadIdx.x >> 5, ln = threadIdx.x & 31;
            for (int kk = w; kk < nk; kk += kColThreads / 32) {
                float qm = -INFINITY, pm = INFINITY;
                bool nan = false;
                for (int cc = ln; cc < TJ; cc += 32) {
                    const float q = s_u[kk][cc];
                    nan |= q != q;
                    qm = fmaxf(qm, q);
                }
                for (int rr = ln; rr < RB; rr += 32) {
                    const float p = s_v[kk][rr];
                    nan |= p != p;
                    pm = fminf(pm, p);
                }
                qm = warp_max(qm);
                pm = -warp_max(-pm);
                nan = __any_sync(0xffffffffu, nan);
                if (ln == 0) {
                    s_qr[kk] = qm;
                    s_one[kk] = !nan && (qm == -INFINITY || pm == INFINITY || qm - pm <= kDcSpread);
                }
            }
        }
        __syncthreads();
        for (int e = threadIdx.x; e < nk * TJ; e += kColThreads) {
            const int kk = e / TJ, cc = e - kk * TJ;
            const float q = s_u[kk][cc];
            s_u[kk][cc] = (s_one[kk] && q != -INFINITY) ? ex2(q - s_qr[kk]) : 0.f;
        }
        for (int e = threadIdx.x; e < nk * RB; e += kColThreads) {
            const int kk = e / RB, rr = e - kk * RB;
            const float p = s_v[kk][rr];
            s_v[kk][rr] = (s_one[kk] && p != INFINITY) ? s_ff[kk][rr] * ex2(s_qr[kk] - p) : 0.f;
        }
        __syncthreads();
        if (colok) {
            for (int kk = 0; kk < nk; ++kk) {
                float gfj[VEC], bcj[VEC];
#pragma unroll
                for (int q = 0; q < VEC; ++q) {
                    gfj[q] = s_gf[kk][ct * VEC + q];
                    bcj[q] = s_bc[kk][ct * VEC + q];
                }
                if (s_one[kk]) {
                    float uj[VEC];
#pragma unroll
                    for (int q = 0; q < VEC; ++q) uj[q] = s_u[kk][ct * VEC + q];
#pragma unroll
                    for (int s = 0; s < kDcRows; ++s) {
                        const int rr = rl + s * kColRL;
                        const float fk = s_hf[kk][rr];
                        const float vi = s_v[kk][rr];
#pragma unroll
                        for (int q = 0; q < VEC; ++q) {
                            const float tc = fmaf(fk - c[s][q], k2, bcj[q]);
                            acc[s][q] = fmaf(fmaf(vi, uj[q], gfj[q]), ex2(tc), acc[s][q]);
                        }
                    }
                } else {
                float gpj[VEC];
#pragma unroll
                for (int q = 0; q < VEC; ++q) gpj[q] = s_hg[kk][ct * VEC + q];
#pragma unroll
                for (int s = 0; s < kDcRows; ++s) {
                    const int rr = rl + s * kColRL;
                    const float fk = s_hf[kk][rr];
                    const float ffk = s_ff[kk][rr];
                    const float ark = s_ar[kk][rr];
#pragma unroll
                    for (int q = 0; q < VEC; ++q) {
                        const float tc = fmaf(fk - c[s][q], k2, bcj[q]);
                        const float tr = fmaf(gpj[q] - c[s][q], k2, ark);
                        acc[s][q] = fmaf(gfj[q], ex2(tc), acc[s][q]);
                        acc[s][q] = fmaf(ffk, ex2(tr), acc[s][q]);
                    }
                }
                }
            }
        }
    }
    if (!colok) return;
#pragma unroll
    for (int s = 0; s < kDcRows; ++s) {
        if (rows[s] >= a.N) continue;
        float* dst = a.dC + (b * a.N + rows[s]) * a.M + j0;
#pragma unroll
        for (int q = 0; q < VEC; ++q)
            if (!(rv[s] && cv[q])) acc[s][q] = 0.f;
        if constexpr (VEC == 4) {
            __stcs(reinterpret_cast<float4*>(dst),
                   make_float4(acc[s][0], acc[s][1], acc[s][2], acc[s][3]));
        } else {
            dst[0] = acc[s][0];
        }
    }
}

// ---------------------------------------------------------------------------
struct BwdWs {
    SolveWs solve;
    float* hf;      // (K+1) x BN
    float* hg;      // (K+1) x BM
    float* lr;      // K x BN  row LSEs
    float* lc;      // K x BM  column LSEs
    float* ff;      // K x BN
    float* ar;      // K x BN
    float* gf;      // K x BM
    float* bc;      // K x BM
    float* Fb;      // BN
    float* Gb;      // BM
    float* Gprev;   // BM
    float* R;       // BN
    float* S;       // BM
    void* band;
    size_t bytes;
};

static BwdWs carve_bwd(void* base, int64_t B, int64_t N, int64_t M, int64_t K) {
    BwdWs w{};
    const size_t solve_bytes = carve_solve(nullptr, B, N, M).bytes;
    char* p = (char*)base;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        char* r = p ? p + off : nullptr;
        off += align_up(bytes);
        return r;
    };
    w.solve = carve_solve(take(solve_bytes), B, N, M);
    const size_t BN = (size_t)(B * N) * sizeof(float), BM = (size_t)(B * M) * sizeof(float);
    w.hf = (float*)take(BN * (K + 1));
    w.hg = (float*)take(BM * (K + 1));
    w.lr = (float*)take(BN * K);
    w.lc = (float*)take(BM * K);
    w.ff = (float*)take(BN * K);
    w.ar = (float*)take(BN * K);
    w.gf = (float*)take(BM * K);
    w.bc = (float*)take(BM * K);
    w.Fb = (float*)take(BN);
    w.Gb = (float*)take(BM);
    w.Gprev = (float*)take(BM);
    w.R = (float*)take(BN);
    w.S = (float*)take(BM);
    w.band = take(band_workspace_bytes(B, N, M));
    w.bytes = off;
    return w;
}

static unsigned blocks_for(int64_t n, int t) { return (unsigned)((n + t - 1) / t); }

}  // namespace sk

using namespace sk;

extern "C" {

size_t sk_backward_workspace_bytes(int64_t B, int64_t N, int64_t M, int64_t K) {
    if (B <= 0 || N <= 0 || M <= 0 || K < 0) return 0;
    return carve_bwd(nullptr, B, N, M, K > 0 ? K : 1).bytes;
}

int sk_backward(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb, int64_t sCn,
                int64_t sCm, const float* a, const float* b, const uint8_t* mask_a,
                const uint8_t* mask_b, double epsilon, double tau_a, double tau_b,
                int max_iters, double threshold, int grad_iters, const float* f_star,
                const float* g_star, const float* grad_f, const float* grad_g, float* dC,
                float* dlog_a, float* dlog_b, void* workspace, size_t workspace_bytes,
                int* K_out, void* stream) {
    clear_error();
    if (int e = check_problem(C, B, N, M, epsilon)) return e;
    if (max_iters < 0) return fail(SK_ERR_ARG, "max_iters must be >= 0");
    if (!dC) return fail(SK_ERR_ARG, "dC must be non-NULL");
    const bool full = !(grad_iters > 0 && grad_iters < max_iters);
    if (!full && (!f_star || !g_star))
        return fail(SK_ERR_ARG, "truncated mode needs f_star and g_star");
    const int Kmax = full ? max_iters : grad_iters;
    const BwdWs w = carve_bwd(workspace, B, N, M, Kmax > 0 ? Kmax : 1);
    if (!workspace || workspace_bytes < w.bytes)
        return fail(SK_ERR_WORKSPACE, "workspace smaller than sk_backward_workspace_bytes");
    cudaStream_t s = (cudaStream_t)stream;
    const Problem P{C, B, N, M, sCb, sCn, sCm};
    const SweepPlan p = make_plan(C, B, N, M, sCb, sCn, sCm);
    const Scalars sc = make_scalars(epsilon, tau_a, tau_b);
    const int64_t BN = B * N, BM = B * M;

    // ---- forward recompute, recording f^k, g^k and the LSEs -------------
    const bool checks = full && threshold > 0.0;
    if (!full) {
        SK_CUDA(cudaMemcpyAsync(w.hf, f_star, sizeof(float) * BN, cudaMemcpyDeviceToDevice, s));
        SK_CUDA(cudaMemcpyAsync(w.hg, g_star, sizeof(float) * BM, cudaMemcpyDeviceToDevice, s));
    }
    if (int e = init_solve(P, w.solve, a, b, mask_a, mask_b, w.hf, w.hg, Kmax,
                           checks ? 1 : 0, (float)threshold, 1, full ? 0 : 1, s,
                           full ? 1 : 0))
        return e;
    const uint8_t* it_ma = full ? mask_a : nullptr;
    const uint8_t* it_mb = full ? mask_b : nullptr;
    // shapes whose forward runs the single-read iteration recompute on it too
    // (one read of C per iteration instead of two), recording the same
    // vectors: the step's rows' LSE and new f, the finish's columns' LSE and
    // new g
    const bool single_read = p.fused != 0;
    for (int it = 0; it < Kmax && single_read; ++it) {
        const StepOut out{w.hf + (int64_t)it * BN, w.hf + (int64_t)(it + 1) * BN,
                          w.lr + (int64_t)it * BN, full ? 1 : 0};
        if (int e = launch_fused(P, p, w.solve, sc, it_ma, out.f_out, s, &out)) return e;
        if (int e = launch_col_finish(w.solve.fparts, (int)p.chunks, B * M + 4, B, M, it_mb,
                                      w.solve.log_b, w.hg + (int64_t)(it + 1) * BM,
                                      w.solve.g_eff, sc, w.solve.status, s,
                                      w.hg + (int64_t)it * BM, w.lc + (int64_t)it * BM,
                                      full ? 1 : 0))
            return e;
    }
    for (int it = 0; it < Kmax && !single_read; ++it) {
        RowArgs ra = make_row_args(P, w.solve, sc, it_ma, w.hf + (int64_t)(it + 1) * BN,
                                   w.hf + (int64_t)it * BN);
        ra.lse_out = w.lr + (int64_t)it * BN;
        ra.guard = full ? 1 : 0;
        if (!full) ra.ranges = nullptr;
        ColArgs ca = make_col_args(P, p, w.solve, sc, it_mb, w.hg + (int64_t)(it + 1) * BM,
                                   w.hg + (int64_t)it * BM);
        ca.lse_out = w.lc + (int64_t)it * BM;
        ca.guard = full ? 1 : 0;
        if (!full) ca.ranges = nullptr;
        launch_row(p, ra, s);
        launch_col(p, ca, s);
        SK_LAUNCHED("backward recompute sweep launch");
    }
    int K = Kmax;
    if (checks) {
        Status hs;
        if (int e = read_status(w.solve.status, &hs, s)) return e;
        K = hs.done ? hs.n_iters : Kmax;
    }
    if (K_out) *K_out = K;

    // ---- reverse sweep --------------------------------------------------
    constexpr int T = 256;
    k_bwd_seed<<<blocks_for(BN, T), T, 0, s>>>(grad_f, mask_a, w.Fb, BN);
    k_bwd_seed<<<blocks_for(BM, T), T, 0, s>>>(grad_g, mask_b, w.Gb, BM);
    if (dlog_a) SK_CUDA(cudaMemsetAsync(dlog_a, 0, sizeof(float) * BN, s));
    if (dlog_b) SK_CUDA(cudaMemsetAsync(dlog_b, 0, sizeof(float) * BM, s));
    SK_LAUNCHED("backward seed launch");
    const bool v4 = p.vec == 4 && ((uintptr_t)dC % 16 == 0);
    // shapes with whole rows in shared memory take each reverse step with one
    // read of C (sk_bwd_rows.cu): the row pass, the row adjoint step and the
    // chunks' column sums in one kernel, then their merge and the column
    // adjoint step of the next step in k_bwd_vec
    const bool single_rev = bwd_rows_shape(p, N, M);
    const int64_t rchunks = single_rev ? bwd_rows_chunks(B, N, M) : 0;
    for (int k = K; k >= 1 && single_rev; --k) {
        BwdVecArgs cv{};
        cv.n = BM;
        cv.mask = mask_b;
        cv.lse = w.lc + (int64_t)(k - 1) * BM;
        cv.adj = w.Gb;
        cv.prev = w.Gprev;
        cv.keep = w.Gprev;
        cv.w_out = w.gf + (int64_t)(k - 1) * BM;
        cv.off_out = w.bc + (int64_t)(k - 1) * BM;
        cv.dlog = dlog_b;
        cv.rho = sc.rho_b;
        cv.omr = sc.omr_b;
        cv.eps = sc.eps;
        cv.full = full;
        cv.parts = w.solve.fparts;
        cv.nparts = (int)rchunks;
        cv.pstride = BM + 4;
        launch_pdl(k_bwd_vec, dim3(blocks_for(BM, T)), dim3(T), 0, s, cv, 1, k == K ? 1 : 0);
        SK_LAUNCHED("k_bwd_vec launch");
        BwdRowsStep r{};
        r.fk = w.hf + (int64_t)k * BN;
        r.gprev = w.hg + (int64_t)(k - 1) * BM;
        r.gf = w.gf + (int64_t)(k - 1) * BM;
        r.bc = w.bc + (int64_t)(k - 1) * BM;
        r.lr = w.lr + (int64_t)(k - 1) * BN;
        r.mask_a = it_ma;
        r.mask_b = it_mb;
        r.Fb = w.Fb;
        r.ff = w.ff + (int64_t)(k - 1) * BN;
        r.ar = w.ar + (int64_t)(k - 1) * BN;
        r.dlog_a = dlog_a;
        r.parts = w.solve.fparts;
        r.pstride = BM + 4;
        r.chunks = rchunks;
        r.k2 = (float)(1.4426950408889634074 / (double)sc.eps);
        r.eps = sc.eps;
        r.rho = sc.rho_a;
        r.omr = sc.omr_a;
        r.full = full ? 1 : 0;
        r.col_pass = k > 1 ? 1 : 0;
        r.status = w.solve.status;
        if (int e = launch_bwd_rows(P, r, s)) return e;
    }
    for (int k = K; k >= 1 && !single_rev; --k) {
        // column half-step adjoint -> gf^k, bc^k, Gprev
        BwdVecArgs cv{};
        cv.n = BM;
        cv.mask = mask_b;
        cv.lse = w.lc + (int64_t)(k - 1) * BM;
        cv.adj = w.Gb;
        cv.sub = w.S;
        cv.prev = w.Gprev;
        cv.keep = w.Gprev;
        cv.w_out = w.gf + (int64_t)(k - 1) * BM;
        cv.off_out = w.bc + (int64_t)(k - 1) * BM;
        cv.dlog = dlog_b;
        cv.rho = sc.rho_b;
        cv.omr = sc.omr_b;
        cv.eps = sc.eps;
        cv.full = full;
        k_bwd_vec<<<blocks_for(BM, T), T, 0, s>>>(cv, 1, k == K);
        SK_LAUNCHED("k_bwd_vec launch");
        // R_i = sum_j gf_j pi_c_ij
        BandArgs br{};
        br.C = C; br.sCb = sCb; br.sCn = sCn; br.sCm = sCm; br.B = B; br.N = N; br.M = M;
        br.u = w.hf + (int64_t)k * BN;
        br.beta = w.bc + (int64_t)(k - 1) * BM;
        br.wc = w.gf + (int64_t)(k - 1) * BM;
        br.mask_a = it_ma;
        br.mask_b = it_mb;
        br.inv_eps = sc.k;
        br.scale = 1.f;
        br.row_q = 2;
        br.row_out0 = w.R;
        br.epi = EPI_RAW;
        if (int e = launch_band(br, p.vec == 4, w.band, s)) return e;
        // row half-step adjoint -> ff^k, ar^k, Fb
        BwdVecArgs rv{};
        rv.n = BN;
        rv.mask = mask_a;
        rv.lse = w.lr + (int64_t)(k - 1) * BN;
        rv.adj = w.Fb;
        rv.sub = w.R;
        rv.w_out = w.ff + (int64_t)(k - 1) * BN;
        rv.off_out = w.ar + (int64_t)(k - 1) * BN;
        rv.dlog = dlog_a;
        rv.rho = sc.rho_a;
        rv.omr = sc.omr_a;
        rv.eps = sc.eps;
        rv.full = full;
        k_bwd_vec<<<blocks_for(BN, T), T, 0, s>>>(rv, 0, 0);
        SK_LAUNCHED("k_bwd_vec launch");
        // S_j = sum_i ff_i pi_r_ij (Gb for step k-1 = Gprev - S)
        BandArgs bc{};
        bc.C = C; bc.sCb = sCb; bc.sCn = sCn; bc.sCm = sCm; bc.B = B; bc.N = N; bc.M = M;
        bc.v = w.hg + (int64_t)(k - 1) * BM;
        bc.alpha = w.ar + (int64_t)(k - 1) * BN;
        bc.wr = w.ff + (int64_t)(k - 1) * BN;
        bc.mask_a = it_ma;
        bc.mask_b = it_mb;
        bc.inv_eps = sc.k;
        bc.scale = 1.f;
        bc.col_q = 2;
        bc.col_out0 = w.S;
        bc.epi = EPI_RAW;
        if (k > 1) {
            if (int e = launch_band(bc, p.vec == 4, w.band, s)) return e;
        }
    }
    // ---- dC in one pass ---------------------------------------------------
    DcArgs da{};
    da.C = C; da.sCb = sCb; da.sCn = sCn; da.sCm = sCm; da.B = B; da.N = N; da.M = M;
    da.K = K;
    da.BN = BN;
    da.BM = BM;
    da.hf = w.hf;
    da.hg = w.hg;
    da.ff = w.ff;
    da.ar = w.ar;
    da.gf = w.gf;
    da.bc = w.bc;
    da.mask_a = it_ma;
    da.mask_b = it_mb;
    da.k2 = (float)(1.4426950408889634074 / (double)sc.eps);
    da.dC = dC;
    const int vec = v4 ? 4 : 1;
    da.ntiles = (M + 32 * vec - 1) / (32 * vec);
    da.nrowblk = (N + kColRL * kDcRows - 1) / (kColRL * kDcRows);
    const int64_t grid = B * da.ntiles * da.nrowblk;
    if (v4) k_bwd_dc<4><<<(unsigned)grid, kColThreads, 0, s>>>(da);
    else k_bwd_dc<1><<<(unsigned)grid, kColThreads, 0, s>>>(da);
    SK_LAUNCHED("k_bwd_dc launch");
    // the single-read kernels' bounded waits record a give-up in the status
    if (single_read || single_rev) {
        Status hs;
        if (int e = read_status(w.solve.status, &hs, s)) return e;
        if (hs.err == 2)
            return fail(SK_ERR_TIMEOUT, "a backward kernel gave up waiting for its copies");
        if (hs.err) return fail(SK_ERR_DEVICE, "a backward kernel reported an error");
    }
    return SK_OK;
}

}  // extern "C"
