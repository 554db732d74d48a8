/*
 * sk_oracle.c -- CPU restatement of the reference Sinkhorn hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the parity oracle: it is linked by
 * the tests, by __graft_entry__.smoke() and by the CPU-baseline leg of
 * bench.py, and by nothing else. The product path (sinkhorn_b200/) never
 * calls it and has no CPU fallback.
 *
 * Parity pin: every function below is checked against golden vectors that
 * tests/golden/make_golden.py produced by running the reference package
 * (vv137/sinkhorn, PyTorch path and, for small shapes, the Triton path under
 * TRITON_INTERPRET=1) on seeded inputs.
 *
 * The file is compiled twice: with REAL=double (prefix sko64_, the parity
 * oracle) and with REAL=float (prefix sko32_, the arithmetic type of the
 * reference, used as the timed CPU baseline). Arrays are dense row-major:
 * C is (B,N,M), row vectors are (B,N), column vectors are (B,M), masks are
 * uint8 (B,N)/(B,M) with NULL meaning "no mask".
 *
 * Reference algorithm followed (paths relative to the reference project):
 *   src/sinkhorn/pytorch/unbalanced.py:13-163   (rho, softmin, main loop)
 *   src/sinkhorn/triton/forward.py:85-186       (10-iteration check cadence)
 *   src/sinkhorn/triton/lse_kernel.py:21-293    (softmin with 0 for empty rows)
 *   src/sinkhorn/autograd.py:61-178             (truncated / full backward)
 *   src/sinkhorn/sinkhorn.py:27-67              (transport_plan, cost)
 *   src/sinkhorn/triton/jvp_kernel.py:113-182   (jvp on a materialised plan)
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifndef REAL
#define REAL double
#endif
#ifndef PFX
#define PFX sko64_
#endif
#define SKO_CAT_(a, b) a##b
#define SKO_CAT(a, b) SKO_CAT_(a, b)
#define FN(name) SKO_CAT(PFX, name)

#ifdef _OPENMP
#include <omp.h>
#endif

/* Threads of the OpenMP regions that follow (the timed CPU baseline uses
 * every host core, whatever OMP_NUM_THREADS a launcher exported). */
void FN(set_threads)(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

#if defined(SKO_REAL_IS_FLOAT)
#define R_EXP expf
#define R_LOG logf
#define R_FABS fabsf
#else
#define R_EXP exp
#define R_LOG log
#define R_FABS fabs
#endif

typedef int64_t i64;

#define COL_BLOCK 64

static inline int valid_row(const uint8_t* mask_a, i64 b, i64 N, i64 i) {
    return mask_a == NULL || mask_a[b * N + i] != 0;
}
static inline int valid_col(const uint8_t* mask_b, i64 b, i64 M, i64 j) {
    return mask_b == NULL || mask_b[b * M + j] != 0;
}

/* torch.logsumexp semantics: shift by the max unless the max is +-inf, in
 * which case the shift is 0 (so an all -inf set gives -inf). */
static inline REAL lse_finish(REAL mx, REAL sum) {
    REAL shift = isinf(mx) ? (REAL)0 : mx;
    return R_LOG(sum) + shift;
}

/*
 * Row softmin for one row: -eps * LSE_j((g_j - C_ij)/eps) over the columns
 * that take part. `use_masks` selects the C_masked semantics of
 * unbalanced.py:118-123 (masked rows and columns behave as C=+inf, i.e. they
 * drop out of the sum). Returns the LSE (natural log); -inf for an empty set.
 */
static REAL row_lse(const REAL* Crow, const REAL* grow, i64 M, REAL eps,
                    const uint8_t* mrow_b /* mask_b row or NULL */) {
    REAL mx = -INFINITY;
    for (i64 j = 0; j < M; ++j) {
        if (mrow_b && !mrow_b[j]) continue;
        REAL x = (grow[j] - Crow[j]) / eps;
        if (x > mx || isnan(x)) mx = x;
    }
    REAL shift = isinf(mx) ? (REAL)0 : mx;
    REAL sum = 0;
    for (i64 j = 0; j < M; ++j) {
        if (mrow_b && !mrow_b[j]) continue;
        REAL x = (grow[j] - Crow[j]) / eps;
        sum += R_EXP(x - shift);
    }
    return lse_finish(mx, sum);
}

/* Column LSEs for one batch item: lse[j] = LSE_i((f_i - C_ij)/eps). */
static void col_lse(const REAL* Cb, const REAL* fb, i64 N, i64 M, REAL eps,
                    const uint8_t* ma /* row mask of this item or NULL */,
                    const uint8_t* mb /* col mask of this item or NULL */,
                    REAL* lse_out) {
#pragma omp parallel for schedule(static)
    for (i64 j0 = 0; j0 < M; j0 += COL_BLOCK) {
        i64 j1 = j0 + COL_BLOCK < M ? j0 + COL_BLOCK : M;
        REAL mx[COL_BLOCK], sm[COL_BLOCK];
        for (i64 j = j0; j < j1; ++j) { mx[j - j0] = -INFINITY; sm[j - j0] = 0; }
        for (i64 i = 0; i < N; ++i) {
            if (ma && !ma[i]) continue;
            const REAL* Crow = Cb + i * M;
            REAL fi = fb[i];
            for (i64 j = j0; j < j1; ++j) {
                REAL x = (fi - Crow[j]) / eps;
                if (x > mx[j - j0] || isnan(x)) mx[j - j0] = x;
            }
        }
        for (i64 i = 0; i < N; ++i) {
            if (ma && !ma[i]) continue;
            const REAL* Crow = Cb + i * M;
            REAL fi = fb[i];
            for (i64 j = j0; j < j1; ++j) {
                REAL shift = isinf(mx[j - j0]) ? (REAL)0 : mx[j - j0];
                REAL x = (fi - Crow[j]) / eps;
                sm[j - j0] += R_EXP(x - shift);
            }
        }
        for (i64 j = j0; j < j1; ++j) {
            if (mb && !mb[j]) { lse_out[j] = -INFINITY; continue; }
            lse_out[j] = lse_finish(mx[j - j0], sm[j - j0]);
        }
    }
}

/* ---------------------------------------------------------------------- */
/* Standalone softmins (lse_kernel.py:210-293): out = -eps*LSE, 0 if empty. */

void FN(lse_row)(const REAL* C, i64 B, i64 N, i64 M, const REAL* g, double eps_d,
                 REAL* out) {
    REAL eps = (REAL)eps_d;
#pragma omp parallel for collapse(2) schedule(static)
    for (i64 b = 0; b < B; ++b)
        for (i64 i = 0; i < N; ++i) {
            REAL l = row_lse(C + (b * N + i) * M, g + b * M, M, eps, NULL);
            out[b * N + i] = (l == -INFINITY) ? (REAL)0 : -eps * l;
        }
}

void FN(lse_col)(const REAL* C, i64 B, i64 N, i64 M, const REAL* f, double eps_d,
                 REAL* out) {
    REAL eps = (REAL)eps_d;
    for (i64 b = 0; b < B; ++b) {
        col_lse(C + b * N * M, f + b * N, N, M, eps, NULL, NULL, out + b * M);
        for (i64 j = 0; j < M; ++j) {
            REAL l = out[b * M + j];
            out[b * M + j] = (l == -INFINITY) ? (REAL)0 : -eps * l;
        }
    }
}

/* ---------------------------------------------------------------------- */
/*
 * One Sinkhorn iteration in the two semantics the reference uses.
 *
 * masked_mode = 1: forward semantics, unbalanced.py:125-149 and
 *   forward.py:14-82,161-171 -- C_masked (+inf fill), the isinf guard on the
 *   softmin, masked_fill(0) of f_new / g_new after both half-steps.
 * masked_mode = 0: the truncated-backward iteration of autograd.py:162-171 --
 *   raw C, no guard, no masking (masks are applied by the caller at the end).
 *
 * Writes f_new/g_new and, if non-NULL, the natural-log LSE vectors used for
 * each half-step (lse_r: (B,N), lse_c: (B,M)); those are -inf for empty sets.
 */
static void iterate_once(const REAL* C, i64 B, i64 N, i64 M,
                         const REAL* log_a, const REAL* log_b,
                         const uint8_t* mask_a, const uint8_t* mask_b,
                         REAL eps, REAL rho_a, REAL rho_b, int masked_mode,
                         const REAL* f, const REAL* g, REAL* f_new, REAL* g_new,
                         REAL* lse_r, REAL* lse_c) {
    const uint8_t* ma_ = masked_mode ? mask_a : NULL;
    const uint8_t* mb_ = masked_mode ? mask_b : NULL;
#pragma omp parallel for collapse(2) schedule(static)
    for (i64 b = 0; b < B; ++b)
        for (i64 i = 0; i < N; ++i) {
            REAL l;
            if (!valid_row(ma_, b, N, i)) l = -INFINITY;
            else l = row_lse(C + (b * N + i) * M, g + b * M, M, eps,
                             mb_ ? mb_ + b * M : NULL);
            if (lse_r) lse_r[b * N + i] = l;
            REAL sm = -eps * l;
            if (masked_mode && isinf(sm)) sm = 0;
            REAL full = eps * log_a[b * N + i] + sm;
            REAL fn = rho_a * f[b * N + i] + ((REAL)1 - rho_a) * full;
            f_new[b * N + i] = fn;
        }
    /* The column half-step reads f_new *before* the row masking of
     * forward.py:168-169, but masked rows are excluded from the column sum in
     * masked mode, so the order does not change any value. */
    for (i64 b = 0; b < B; ++b) {
        REAL* lc = (REAL*)malloc(sizeof(REAL) * (size_t)M);
        col_lse(C + b * N * M, f_new + b * N, N, M, eps,
                ma_ ? ma_ + b * N : NULL, mb_ ? mb_ + b * M : NULL, lc);
        for (i64 j = 0; j < M; ++j) {
            if (lse_c) lse_c[b * M + j] = lc[j];
            REAL sm = -eps * lc[j];
            if (masked_mode && isinf(sm)) sm = 0;
            REAL full = eps * log_b[b * M + j] + sm;
            g_new[b * M + j] = rho_b * g[b * M + j] + ((REAL)1 - rho_b) * full;
        }
        free(lc);
    }
    if (masked_mode) {
        if (mask_a)
            for (i64 t = 0; t < B * N; ++t) if (!mask_a[t]) f_new[t] = 0;
        if (mask_b)
            for (i64 t = 0; t < B * M; ++t) if (!mask_b[t]) g_new[t] = 0;
    }
}

/*
 * Forward solve (sinkhorn_unbalanced / sinkhorn_forward_triton). f and g are
 * in/out (the reference starts from zeros; the caller zeroes them).
 * check_every = 1 reproduces unbalanced.py:152-161, check_every = 10
 * reproduces forward.py:176-182. Convergence: max over the whole batch of
 * max|f_new - f| and max|g_new - g| strictly below `threshold`.
 * Returns the number of iterations run.
 */
int FN(forward)(const REAL* C, i64 B, i64 N, i64 M, const REAL* log_a,
                const REAL* log_b, const uint8_t* mask_a, const uint8_t* mask_b,
                double eps_d, double rho_a_d, double rho_b_d, int max_iters,
                double threshold, int check_every, REAL* f, REAL* g,
                int* converged_out) {
    REAL eps = (REAL)eps_d, rho_a = (REAL)rho_a_d, rho_b = (REAL)rho_b_d;
    REAL* fn = (REAL*)malloc(sizeof(REAL) * (size_t)(B * N));
    REAL* gn = (REAL*)malloc(sizeof(REAL) * (size_t)(B * M));
    int n_iters = 0, converged = 0;
    if (check_every < 1) check_every = 1;
    for (int it = 0; it < max_iters; ++it) {
        iterate_once(C, B, N, M, log_a, log_b, mask_a, mask_b, eps, rho_a, rho_b,
                     1, f, g, fn, gn, NULL, NULL);
        n_iters = it + 1;
        int stop = 0;
        if ((it + 1) % check_every == 0) {
            double fd = 0, gd = 0;
            for (i64 t = 0; t < B * N; ++t) {
                double d = fabs((double)fn[t] - (double)f[t]);
                if (d > fd || isnan(d)) fd = d;
            }
            for (i64 t = 0; t < B * M; ++t) {
                double d = fabs((double)gn[t] - (double)g[t]);
                if (d > gd || isnan(d)) gd = d;
            }
            double res = fd > gd ? fd : gd;
            if (res < threshold) { converged = 1; stop = 1; }
        }
        memcpy(f, fn, sizeof(REAL) * (size_t)(B * N));
        memcpy(g, gn, sizeof(REAL) * (size_t)(B * M));
        if (stop) break;
    }
    free(fn);
    free(gn);
    if (converged_out) *converged_out = converged;
    return n_iters;
}

/*
 * n Gauss-Seidel iterations from the potentials already in (f, g), in place,
 * with no convergence check.
 * masked_mode = 0 restates _sinkhorn_iters_from_init (autograd.py:134-178):
 *   raw C (no +inf fill), no isinf guard on the softmins, and masked_fill(0)
 *   of the final f / g only (autograd.py:173-176).
 * masked_mode = 1 runs the forward iteration (unbalanced.py:125-149,
 *   forward.py:161-171) n times, as the forward solve does between checks.
 */
void FN(iterate)(const REAL* C, i64 B, i64 N, i64 M, const REAL* log_a, const REAL* log_b,
                 const uint8_t* mask_a, const uint8_t* mask_b, double eps_d, double rho_a_d,
                 double rho_b_d, int masked_mode, int n, REAL* f, REAL* g) {
    REAL eps = (REAL)eps_d, rho_a = (REAL)rho_a_d, rho_b = (REAL)rho_b_d;
    REAL* fn = (REAL*)malloc(sizeof(REAL) * (size_t)(B * N));
    REAL* gn = (REAL*)malloc(sizeof(REAL) * (size_t)(B * M));
    for (int it = 0; it < n; ++it) {
        iterate_once(C, B, N, M, log_a, log_b, mask_a, mask_b, eps, rho_a, rho_b,
                     masked_mode, f, g, fn, gn, NULL, NULL);
        memcpy(f, fn, sizeof(REAL) * (size_t)(B * N));
        memcpy(g, gn, sizeof(REAL) * (size_t)(B * M));
    }
    if (!masked_mode) {
        if (mask_a)
            for (i64 t = 0; t < B * N; ++t) if (!mask_a[t]) f[t] = 0;
        if (mask_b)
            for (i64 t = 0; t < B * M; ++t) if (!mask_b[t]) g[t] = 0;
    }
    free(fn);
    free(gn);
}

/* ---------------------------------------------------------------------- */
/*
 * Backward of SinkhornFunction (autograd.py:61-131), reverse mode written out
 * by hand. Let pi_r[i,j] = exp((g^{k-1}_j - C_ij)/eps - lse_r^k_i) and
 * pi_c[i,j] = exp((f^k_i - C_ij)/eps - lse_c^k_j). Going backwards over the
 * K recorded iterations, with adjoints Fb (of f^k) and Gb (of g^k):
 *   gf = (1-rho_b) Gb^k ;  Fb^k_i -= sum_j gf_j pi_c ;  dC += gf_j pi_c
 *   ff = (1-rho_a) Fb^k ;  Gb^{k-1}_j = rho_b Gb^k_j - sum_i ff_i pi_r
 *   Fb^{k-1} = rho_a Fb^k ; dC += ff_i pi_r ; dlog_a += eps ff ; dlog_b += eps gf
 * In full mode (grad_iters outside (0, max_iters)) the recorded iterations are
 * a fresh masked solve from zeros with a per-iteration convergence check
 * (autograd.py:98-113): adjoints are zeroed at masked rows/columns before each
 * half-step (masked_fill backward), masked entries of C get no gradient and a
 * guarded (empty) softmin passes no gradient. In truncated mode
 * (0 < grad_iters < max_iters) the K iterations start from (f*, g*) on raw C
 * with masks applied only to the final potentials (autograd.py:134-178).
 *
 * Outputs dC (B,N,M), dlog_a (B,N), dlog_b (B,M). Returns K.
 */
int FN(backward)(const REAL* C, i64 B, i64 N, i64 M, const REAL* log_a,
                 const REAL* log_b, const uint8_t* mask_a, const uint8_t* mask_b,
                 double eps_d, double rho_a_d, double rho_b_d, int full_mode,
                 int grad_iters, int max_iters, double threshold,
                 const REAL* f_star, const REAL* g_star, const REAL* grad_f,
                 const REAL* grad_g, REAL* dC, REAL* dlog_a, REAL* dlog_b) {
    REAL eps = (REAL)eps_d, rho_a = (REAL)rho_a_d, rho_b = (REAL)rho_b_d;
    int Kmax = full_mode ? max_iters : grad_iters;
    i64 BN = B * N, BM = B * M;
    REAL* fh = (REAL*)calloc((size_t)((Kmax + 1) * BN), sizeof(REAL));
    REAL* gh = (REAL*)calloc((size_t)((Kmax + 1) * BM), sizeof(REAL));
    REAL* lr = (REAL*)calloc((size_t)((Kmax + 1) * BN), sizeof(REAL));
    REAL* lc = (REAL*)calloc((size_t)((Kmax + 1) * BM), sizeof(REAL));
    int K = 0;
    if (!full_mode) {
        memcpy(fh, f_star, sizeof(REAL) * (size_t)BN);
        memcpy(gh, g_star, sizeof(REAL) * (size_t)BM);
    }
    for (int it = 0; it < Kmax; ++it) {
        REAL* f0 = fh + (i64)it * BN; REAL* g0 = gh + (i64)it * BM;
        REAL* f1 = fh + (i64)(it + 1) * BN; REAL* g1 = gh + (i64)(it + 1) * BM;
        iterate_once(C, B, N, M, log_a, log_b, mask_a, mask_b, eps, rho_a, rho_b,
                     full_mode, f0, g0, f1, g1, lr + (i64)(it + 1) * BN,
                     lc + (i64)(it + 1) * BM);
        K = it + 1;
        if (full_mode) {
            double res = 0;
            for (i64 t = 0; t < BN; ++t) {
                double d = fabs((double)f1[t] - (double)f0[t]);
                if (d > res || isnan(d)) res = d;
            }
            for (i64 t = 0; t < BM; ++t) {
                double d = fabs((double)g1[t] - (double)g0[t]);
                if (d > res || isnan(d)) res = d;
            }
            if (res < threshold) break;
        }
    }
    REAL* Fb = (REAL*)calloc((size_t)BN, sizeof(REAL));
    REAL* Gb = (REAL*)calloc((size_t)BM, sizeof(REAL));
    REAL* Gprev = (REAL*)calloc((size_t)BM, sizeof(REAL));
    REAL* ff = (REAL*)calloc((size_t)BN, sizeof(REAL));
    REAL* gf = (REAL*)calloc((size_t)BM, sizeof(REAL));
    for (i64 t = 0; t < BN; ++t) Fb[t] = (mask_a && !mask_a[t]) ? 0 : grad_f[t];
    for (i64 t = 0; t < BM; ++t) Gb[t] = (mask_b && !mask_b[t]) ? 0 : grad_g[t];
    memset(dC, 0, sizeof(REAL) * (size_t)(BN * M));
    memset(dlog_a, 0, sizeof(REAL) * (size_t)BN);
    memset(dlog_b, 0, sizeof(REAL) * (size_t)BM);
    const uint8_t* ma_ = full_mode ? mask_a : NULL;
    const uint8_t* mb_ = full_mode ? mask_b : NULL;
    for (int k = K; k >= 1; --k) {
        const REAL* fk = fh + (i64)k * BN;
        const REAL* gkm1 = gh + (i64)(k - 1) * BM;
        const REAL* lrk = lr + (i64)k * BN;
        const REAL* lck = lc + (i64)k * BM;
        /* g^k half-step */
        for (i64 t = 0; t < BM; ++t) {
            REAL gbar = (mb_ && !mb_[t]) ? 0 : Gb[t];
            /* guarded softmin (empty column) passes no gradient */
            int guarded = full_mode && isinf(lck[t]);
            gf[t] = guarded ? 0 : ((REAL)1 - rho_b) * gbar;
            dlog_b[t] += eps * ((REAL)1 - rho_b) * gbar;
            Gprev[t] = rho_b * gbar;
        }
#pragma omp parallel for collapse(2) schedule(static)
        for (i64 b = 0; b < B; ++b)
            for (i64 i = 0; i < N; ++i) {
                if (!valid_row(ma_, b, N, i)) continue;
                const REAL* Crow = C + (b * N + i) * M;
                REAL* dCrow = dC + (b * N + i) * M;
                REAL acc = 0;
                for (i64 j = 0; j < M; ++j) {
                    if (!valid_col(mb_, b, M, j)) continue;
                    REAL w = gf[b * M + j];
                    if (w == 0) continue;
                    REAL p = R_EXP((fk[b * N + i] - Crow[j]) / eps - lck[b * M + j]);
                    acc += w * p;
                    dCrow[j] += w * p;
                }
                Fb[b * N + i] -= acc;
            }
        /* f^k half-step */
        for (i64 t = 0; t < BN; ++t) {
            REAL fbar = (ma_ && !ma_[t]) ? 0 : Fb[t];
            int guarded = full_mode && isinf(lrk[t]);
            ff[t] = guarded ? 0 : ((REAL)1 - rho_a) * fbar;
            dlog_a[t] += eps * ((REAL)1 - rho_a) * fbar;
            Fb[t] = rho_a * fbar;
        }
#pragma omp parallel for collapse(2) schedule(static)
        for (i64 b = 0; b < B; ++b)
            for (i64 j0 = 0; j0 < M; j0 += COL_BLOCK) {
                i64 j1 = j0 + COL_BLOCK < M ? j0 + COL_BLOCK : M;
                for (i64 i = 0; i < N; ++i) {
                    if (!valid_row(ma_, b, N, i)) continue;
                    REAL w = ff[b * N + i];
                    if (w == 0) continue;
                    const REAL* Crow = C + (b * N + i) * M;
                    REAL* dCrow = dC + (b * N + i) * M;
                    for (i64 j = j0; j < j1; ++j) {
                        if (!valid_col(mb_, b, M, j)) continue;
                        REAL p = R_EXP((gkm1[b * M + j] - Crow[j]) / eps - lrk[b * N + i]);
                        Gprev[b * M + j] -= w * p;
                        dCrow[j] += w * p;
                    }
                }
            }
        memcpy(Gb, Gprev, sizeof(REAL) * (size_t)BM);
    }
    free(fh); free(gh); free(lr); free(lc);
    free(Fb); free(Gb); free(Gprev); free(ff); free(gf);
    return K;
}

/* ---------------------------------------------------------------------- */
/* transport_plan (sinkhorn.py:27-54): P = exp((f+g-C)/eps), 0 where masked. */
void FN(plan)(const REAL* C, i64 B, i64 N, i64 M, const REAL* f, const REAL* g,
              double eps_d, const uint8_t* mask_a, const uint8_t* mask_b, REAL* P) {
    REAL eps = (REAL)eps_d;
#pragma omp parallel for collapse(2) schedule(static)
    for (i64 b = 0; b < B; ++b)
        for (i64 i = 0; i < N; ++i) {
            int ra = valid_row(mask_a, b, N, i);
            for (i64 j = 0; j < M; ++j) {
                i64 e = (b * N + i) * M + j;
                if (!ra || !valid_col(mask_b, b, M, j)) { P[e] = 0; continue; }
                P[e] = R_EXP((f[b * N + i] + g[b * M + j] - C[e]) / eps);
            }
        }
}

/* cost (sinkhorn.py:56-67): sum_ij P_ij C_ij with the unmasked plan. */
void FN(cost)(const REAL* C, i64 B, i64 N, i64 M, const REAL* f, const REAL* g,
              double eps_d, REAL* out) {
    REAL eps = (REAL)eps_d;
    for (i64 b = 0; b < B; ++b) {
        double acc = 0;
#pragma omp parallel for reduction(+ : acc) schedule(static)
        for (i64 i = 0; i < N; ++i)
            for (i64 j = 0; j < M; ++j) {
                i64 e = (b * N + i) * M + j;
                REAL p = R_EXP((f[b * N + i] + g[b * M + j] - C[e]) / eps);
                acc += (double)(p * C[e]);
            }
        out[b] = (REAL)acc;
    }
}

/*
 * jvp on a materialised plan (jvp_kernel.py:113-182):
 *   out_f = (P v_g) / max(P 1, 1e-38),  out_g = (P^T v_f) / max(P^T 1, 1e-38),
 * then out = rho*v + (1-rho)*out when rho != 0.
 */
void FN(jvp)(const REAL* P, i64 B, i64 N, i64 M, const REAL* v_f, const REAL* v_g,
             double rho_a_d, double rho_b_d, REAL* out_f, REAL* out_g) {
    REAL rho_a = (REAL)rho_a_d, rho_b = (REAL)rho_b_d;
    const REAL tiny = (REAL)1e-38f;
    for (i64 b = 0; b < B; ++b) {
        for (i64 i = 0; i < N; ++i) {
            REAL pv = 0, rs = 0;
            for (i64 j = 0; j < M; ++j) {
                REAL p = P[(b * N + i) * M + j];
                pv += p * v_g[b * M + j];
                rs += p;
            }
            if (rs < tiny) rs = tiny;
            REAL r = pv / rs;
            if (rho_a != 0) r = rho_a * v_f[b * N + i] + ((REAL)1 - rho_a) * r;
            out_f[b * N + i] = r;
        }
        for (i64 j = 0; j < M; ++j) {
            REAL pv = 0, cs = 0;
            for (i64 i = 0; i < N; ++i) {
                REAL p = P[(b * N + i) * M + j];
                pv += p * v_f[b * N + i];
                cs += p;
            }
            if (cs < tiny) cs = tiny;
            REAL r = pv / cs;
            if (rho_b != 0) r = rho_b * v_g[b * M + j] + ((REAL)1 - rho_b) * r;
            out_g[b * M + j] = r;
        }
    }
}
