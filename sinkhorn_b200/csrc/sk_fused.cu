// sk_fused.cu -- the single-read iteration as one step per launch (the
// kernel is in sk_fused_kernel.cuh), and the plan of the single-read shapes:
// which kernel, how many row chunks, and whether sk_forward may run the whole
// solve as one persistent launch (sk_fused_solve.cu).
#include <algorithm>
#include <cmath>

#include "sk_fused_kernel.cuh"
#include "sk_internal.h"
#include "sk_solve.cuh"

namespace sk {

// One step: grid = CL CTAs per unit (compile-time cluster dims), launched as
// a programmatic dependent of the previous kernel on the stream.
template <int G4, int CL, typename T>
static int launch_step_g(const FusedArgs& a, int64_t nunits, cudaStream_t s) {
    const int64_t part = a.M / CL;
    const size_t smem = fz_smem<CL, T>(part);
    const dim3 grid((unsigned)(CL * nunits));
    if (part == (int64_t)kFzGroup * 4 * G4) {
        if (int e = fz_prepare<G4, true, CL, false, T>()) return e;
        launch_pdl(k_fused_iter<G4, true, CL, false, T>, grid, dim3(kFzThreads), smem, s, a);
    } else {
        if (int e = fz_prepare<G4, false, CL, false, T>()) return e;
        launch_pdl(k_fused_iter<G4, false, CL, false, T>, grid, dim3(kFzThreads), smem, s, a);
    }
    SK_LAUNCHED("k_fused_iter launch");
    return SK_OK;
}

// Co-resident clusters of k_fused_iter with cluster size CL on the current
// device (cached per device; one CTA per SM): ~74 2-CTA clusters on B200.
// 0 when it cannot be queried (no device).
int64_t fz_active_clusters(int CL) {
    static thread_local int cache[64][4] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return 0;
    }
    const int slot = CL == 1 ? 3 : (CL == 2 ? 0 : (CL == 4 ? 1 : 2));
    if (cache[dev][slot] != 0) return cache[dev][slot] > 0 ? cache[dev][slot] : 0;
    int n = 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)CL, 1, 1);
    cfg.blockDim = dim3(kFzThreads, 1, 1);
    cudaError_t e = cudaErrorInvalidValue;
    if (CL == 1 && fz_prepare<8, true, 1, false, float>() == SK_OK) {
        cfg.dynamicSmemBytes = fz_smem<1, float>(kFzMaxPart);
        e = cudaOccupancyMaxActiveClusters(&n, k_fused_iter<8, true, 1, false, float>, &cfg);
    } else if (CL == 2 && fz_prepare<8, true, 2, false, float>() == SK_OK) {
        cfg.dynamicSmemBytes = fz_smem<2, float>(kFzMaxPart);
        e = cudaOccupancyMaxActiveClusters(&n, k_fused_iter<8, true, 2, false, float>, &cfg);
    } else if (CL == 4 && fz_prepare<8, true, 4, false, float>() == SK_OK) {
        cfg.dynamicSmemBytes = fz_smem<4, float>(kFzMaxPart);
        e = cudaOccupancyMaxActiveClusters(&n, k_fused_iter<8, true, 4, false, float>, &cfg);
    } else if (CL == 8 && fz_prepare<8, true, 8, false, float>() == SK_OK) {
        cfg.dynamicSmemBytes = fz_smem<8, float>(kFzMaxPart);
        e = cudaOccupancyMaxActiveClusters(&n, k_fused_iter<8, true, 8, false, float>, &cfg);
    }
    cudaGetLastError();
    if (e != cudaSuccess || n <= 0) n = -1;
    cache[dev][slot] = n;
    return n > 0 ? n : 0;
}

// One-CTA units for 2048 < M < 8192: a CTA holds the whole row (up to 8192
// columns, 16-byte rows), so the per-row pair stays in the CTA; on 2-CTA
// clusters a CTA would hold 1024-4095 columns and the per-row exchange
// dominated (measured slower than the two sweeps).
static bool single_cta_shape(int64_t M) { return M > 2048 && M < 8192 && M % 4 == 0; }

static bool fused_shape(int64_t N, int64_t M) {
    return (fz_cluster_size(M) > 0 || single_cta_shape(M)) && N >= 1;
}

static int64_t fused_min_chunks(int64_t N, int CL) {
    const int64_t mr = CL <= 2 ? fz_max_rows<2>() : fz_max_rows<4>();
    return (N + mr - 1) / mr;
}

// Device-independent bound of the chunks any plan uses (workspace sizing):
// one wave holds at most 148 / CL clusters.
int64_t fused_max_chunks(int64_t B, int64_t N, int64_t M) {
    if (row_warps_shape(N, M)) return row_warps_max_chunks(B, N);
    if (rows_fused_shape(N, M)) return rows_fused_max_chunks(B, N);
    if (!fused_shape(N, M)) return 0;
    const int CL = single_cta_shape(M) ? 1 : fz_cluster_size(M);
    const int64_t wave = std::max<int64_t>(1, (148 / CL) / std::max<int64_t>(B, 1));
    int64_t c = std::min<int64_t>(std::max(fused_min_chunks(N, CL), wave), N);
    if (CL == 2) c = std::max(c, B >= 296 ? (int64_t)1 : (296 + B - 1) / B);
    if (CL == 1) c = std::max(c, B >= 592 ? (int64_t)1 : (592 + B - 1) / B);
    return std::min(c, N);
}

void plan_fused(SweepPlan& p, int64_t B, int64_t N, int64_t M, bool single_cta) {
    p.fused = 0;
    p.fused_ok = 0;
    p.fused_rows = 0;
    p.cluster = 0;
    p.persist = 0;
    p.solve_chunks = 0;
    p.solve_rows = 0;
    if (row_warps_shape(N, M)) {
        // a whole row per warp (k_row_warps): measured per iteration against
        // k_rows_fused, B=64 N=M=1024 with prefix masks 0.063 vs 0.085 ms,
        // B=32 N=M=1024 0.052 vs 0.055 ms (k_rows_fused keeps M = 512 and
        // M > 1024, where it measured faster)
        const int64_t c = row_warps_chunks(B, N);
        p.rows_per_chunk = (N + c - 1) / c;
        p.chunks = c;
        p.fused_ok = 1;
        p.fused_rows = 2;
        p.fused = B * N >= 148 * 32 ? 1 : 0;
        return;
    }
    if (rows_fused_shape(N, M)) {
        // whole rows per CTA (k_rows_fused)
        const int64_t c = rows_fused_chunks(B, N);
        p.rows_per_chunk = (N + c - 1) / c;
        p.chunks = (N + p.rows_per_chunk - 1) / p.rows_per_chunk;
        p.fused_ok = 1;
        p.fused_rows = 1;
        // sk_forward takes it where every SM gets rows to pipeline (measured
        // per iteration against the two sweeps: B=16 N=M=2048 0.078 vs 0.118
        // ms; B=64 N=M=1024 with prefix masks 0.101 vs 0.123 ms); a small batch
        // keeps the sweeps, which spread rows and columns over all SMs
        p.fused = B * N >= 148 * 32 ? 1 : 0;
        return;
    }
    if (!fused_shape(N, M)) return;
    const int CL = (single_cta && single_cta_shape(M)) ? 1 : fz_cluster_size(M);
    if (CL == 0) return;  // (a 16-byte row that 2-CTA clusters cannot halve)
    p.cluster = CL;
    const int64_t Aq = fz_active_clusters(CL);  // 0 without a device
    const int64_t A = Aq > 0 ? Aq : 148 / CL;
    const int64_t max_rows = CL <= 2 ? fz_max_rows<2>() : fz_max_rows<4>();
    // the persistent solve: every unit on its own co-resident cluster (of
    // two or more CTAs)
    if (CL > 1 && Aq > 0 && B <= Aq) {
        const int64_t c = std::min<int64_t>(Aq / B, N);
        const int64_t rpc = (N + c - 1) / c;
        if (rpc <= max_rows) {
            p.persist = 1;
            p.solve_rows = rpc;
            p.solve_chunks = (N + rpc - 1) / rpc;
        }
    }
    if (CL > 2) {
        // 4- and 8-CTA clusters: each CTA holds 4096-8192 columns of a row,
        // as at M = 16384, so sk_forward always takes the single read
        const int64_t c = std::min<int64_t>(std::max(fused_min_chunks(N, CL), A / B), N);
        p.rows_per_chunk = (N + c - 1) / c;
        p.chunks = (N + p.rows_per_chunk - 1) / p.rows_per_chunk;
        if (p.persist) {
            p.chunks = p.solve_chunks;
            p.rows_per_chunk = p.solve_rows;
        }
        p.fused_ok = 1;
        p.fused = 1;
        return;
    }
    const int64_t cmin = fused_min_chunks(N, CL);
    const int64_t cmax = fused_max_chunks(B, N, M);
    int64_t best_c = cmin;
    double best_eff = -1.0;
    auto fill = [&](int64_t c) {
        const int64_t units = B * c;
        const int64_t waves = (units + A - 1) / A;
        return (double)units / (double)(A * waves);
    };
    for (int64_t c = cmin; c <= cmax; ++c) {
        if (c > cmin && N / c < 16) break;  // keep chunks at least 16 rows deep
        const double eff = fill(c);
        if (eff > best_eff + 1e-9) {
            best_eff = eff;
            best_c = c;
        }
    }
    if (CL == 1 && N / best_c < 256) {
        // short one-CTA chunks: every unit pays a ring fill, so the fewest
        // chunks that fill the SMs within 5% of the best (measured B=16
        // N=2048 M=2560: 9 chunks 127 us, 37 chunks 144 us per iteration)
        for (int64_t c = cmin; c < best_c; ++c)
            if (fill(c) >= best_eff - 0.05) {
                best_c = c;
                break;
            }
    }
    p.rows_per_chunk = (N + best_c - 1) / best_c;
    p.chunks = (N + p.rows_per_chunk - 1) / p.rows_per_chunk;
    if (p.persist) {
        // steps chunk like the persistent solve: the same partials merged in
        // the same order, so both give bit-identical potentials
        p.chunks = p.solve_chunks;
        p.rows_per_chunk = p.solve_rows;
    }
    p.fused_ok = 1;
    // sk_forward takes the fused iteration where it measured faster on B200
    // (per iteration, fused vs row + column sweep): N=M=16384 0.203 vs 0.383
    // ms, 8192 0.094 vs 0.125, N=4096 M=16384 0.080 vs 0.120. Below M = 8192
    // a thread folds 8 or fewer columns of a row and the per-row exchange
    // dominates (N=65536 M=4096: 0.464 vs 0.395), so those shapes keep the two
    // sweeps; their fused iteration stays available through
    // sk_solver_fused_step / _finish. (M <= 2048 takes k_rows_fused above.)
    p.fused = (M >= 8192 || CL == 1) ? 1 : 0;
}

FusedArgs fused_args(const Problem& P, const SolveWs& w, const Scalars& sc,
                     const uint8_t* mask_a, float* f, int64_t chunks, int64_t rows_per_chunk) {
    FusedArgs a{};
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
    a.parts = w.fparts;
    a.chunks = chunks;
    a.rows_per_chunk = rows_per_chunk;
    a.k2 = (float)(1.4426950408889634074 / (double)sc.eps);
    a.eps = sc.eps;
    a.rho = sc.rho_a;
    a.omr = sc.omr_a;
    a.st = (Status*)w.status;
    a.lse_out = nullptr;
    a.guard = 1;
    return a;
}

int launch_fused(const Problem& P, const SweepPlan& p, const SolveWs& w, const Scalars& sc,
                 const uint8_t* mask_a, float* f, cudaStream_t s, const StepOut* out) {
    if (p.fused_rows == 2) return launch_row_warps(P, p, w, sc, mask_a, f, s, out);
    if (p.fused_rows) return launch_rows_fused(P, p, w, sc, mask_a, f, s, out);
    FusedArgs a = fused_args(P, w, sc, mask_a, f, p.chunks, p.rows_per_chunk);
    if (out) {
        a.f_in = out->f_in;
        a.f_out = out->f_out;
        a.lse_out = out->lse_out;
        a.guard = out->guard;
    }
    const int64_t nunits = P.B * p.chunks;
    if (p.cluster == 1) {
        // whole rows: (M/4 float4 groups over 256 lanes)
        if (P.M <= 4096) return launch_step_g<4, 1, float>(a, nunits, s);
        return launch_step_g<8, 1, float>(a, nunits, s);
    }
    if (p.cluster == 4) return launch_step_g<8, 4, float>(a, nunits, s);
    if (p.cluster == 8) return launch_step_g<8, 8, float>(a, nunits, s);
    const int64_t g4 = (P.M / 8 + kFzGroup - 1) / kFzGroup;  // float4 groups per thread
    if (p.bf16) {
        if (g4 <= 1) return launch_step_g<1, 2, uint16_t>(a, nunits, s);
        if (g4 <= 2) return launch_step_g<2, 2, uint16_t>(a, nunits, s);
        if (g4 <= 4) return launch_step_g<4, 2, uint16_t>(a, nunits, s);
        return launch_step_g<8, 2, uint16_t>(a, nunits, s);
    }
    if (g4 <= 1) return launch_step_g<1, 2, float>(a, nunits, s);
    if (g4 <= 2) return launch_step_g<2, 2, float>(a, nunits, s);
    if (g4 <= 4) return launch_step_g<4, 2, float>(a, nunits, s);
    return launch_step_g<8, 2, float>(a, nunits, s);
}

}  // namespace sk

using namespace sk;

extern "C" {

int sk_plan_query(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb, int64_t sCn,
                  int64_t sCm, int* vec, int* fused, int64_t* chunks) {
    if (int e = check_problem(C, B, N, M, 1.0)) return e;
    const SweepPlan p = make_plan(C, B, N, M, sCb, sCn, sCm);
    if (vec) *vec = p.vec;
    if (fused) *fused = p.fused ? (p.persist ? 3 : 2) : (p.fused_ok ? 1 : 0);
    if (chunks) *chunks = p.chunks;
    return SK_OK;
}

int sk_solver_fused_step(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                         int64_t sCn, int64_t sCm, const uint8_t* mask_a, double epsilon,
                         double tau_a, float* f, void* workspace, size_t workspace_bytes,
                         void* stream) {
    if (int e = check_problem(C, B, N, M, epsilon)) return e;
    if (!f) return fail(SK_ERR_ARG, "f must be non-NULL");
    const SolveWs w = carve_solve(workspace, B, N, M);
    if (!workspace || workspace_bytes < w.bytes)
        return fail(SK_ERR_WORKSPACE, "workspace smaller than sk_forward_workspace_bytes");
    const Problem P{C, B, N, M, sCb, sCn, sCm};
    const SweepPlan p = make_plan(C, B, N, M, sCb, sCn, sCm);
    if (!p.fused_ok) return fail(SK_ERR_LAYOUT, "this shape / layout has no fused iteration");
    const Scalars sc = make_scalars(epsilon, tau_a, INFINITY);
    return launch_fused(P, p, w, sc, mask_a, f, (cudaStream_t)stream);
}

int sk_solver_fused_finish(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                           int64_t sCn, int64_t sCm, const uint8_t* mask_b, double epsilon,
                           double tau_b, float* g, void* workspace, size_t workspace_bytes,
                           void* stream) {
    if (int e = check_problem(C, B, N, M, epsilon)) return e;
    if (!g) return fail(SK_ERR_ARG, "g must be non-NULL");
    const SolveWs w = carve_solve(workspace, B, N, M);
    if (!workspace || workspace_bytes < w.bytes)
        return fail(SK_ERR_WORKSPACE, "workspace smaller than sk_forward_workspace_bytes");
    const SweepPlan p = make_plan(C, B, N, M, sCb, sCn, sCm);
    if (!p.fused_ok) return fail(SK_ERR_LAYOUT, "this shape / layout has no fused iteration");
    const Scalars sc = make_scalars(epsilon, INFINITY, tau_b);
    return launch_col_finish(w.fparts, (int)p.chunks, B * M + 4, B, M, mask_b, w.log_b, g,
                             w.g_eff, sc, w.status, (cudaStream_t)stream);
}

}  // extern "C"
