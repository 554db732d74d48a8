// sk_fused_solve.cu -- the whole forward solve as one persistent launch of
// the single-read iteration (k_fused_iter<..., PERSIST = true>, see
// sk_fused_kernel.cuh): every unit of the problem on its own co-resident
// cluster, launched cooperatively so that the grid barriers between the
// iterations' phases cannot wait for a CTA that is not running.
#include <cmath>

#include "sk_fused_kernel.cuh"
#include "sk_internal.h"
#include "sk_solve.cuh"

namespace sk {

template <int G4, bool FULL, int CL>
static int launch_solve_t(const FusedArgs& a, int64_t units, cudaStream_t s) {
    if (int e = fz_prepare<G4, FULL, CL, true, float>()) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(CL * units), 1, 1);
    cfg.blockDim = dim3(kFzThreads, 1, 1);
    cfg.dynamicSmemBytes = fz_smem<CL, float>(a.M / CL);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, k_fused_iter<G4, FULL, CL, true, float>, a);
    if (e != cudaSuccess) return cuda_fail(e, "k_fused_iter (persistent solve) launch");
    return SK_OK;
}

// G4 float4 groups per lane cover up to 1024 G4 columns; FULL (no bounds
// guards) only where the row part is exactly that many columns.
template <int CL>
static int launch_solve_cl(const FusedArgs& a, int64_t units, cudaStream_t s) {
    const int64_t part = a.M / CL;
    if constexpr (CL == 2) {
        if (part <= 1024)
            return part == 1024 ? launch_solve_t<1, true, 2>(a, units, s)
                                : launch_solve_t<1, false, 2>(a, units, s);
        if (part <= 2048)
            return part == 2048 ? launch_solve_t<2, true, 2>(a, units, s)
                                : launch_solve_t<2, false, 2>(a, units, s);
        if (part <= 4096)
            return part == 4096 ? launch_solve_t<4, true, 2>(a, units, s)
                                : launch_solve_t<4, false, 2>(a, units, s);
    }
    if (part > kFzMaxPart) return fail(SK_ERR_LAYOUT, "row part above 8192 columns");
    return part == kFzMaxPart ? launch_solve_t<8, true, CL>(a, units, s)
                              : launch_solve_t<8, false, CL>(a, units, s);
}

int launch_fused_solve(const Problem& P, const SweepPlan& p, const SolveWs& w,
                       const Scalars& sc, const uint8_t* mask_a, const uint8_t* mask_b,
                       float* f, float* g, cudaStream_t s) {
    if (!p.persist) return fail(SK_ERR_LAYOUT, "no persistent solve for this shape");
    FusedArgs a = fused_args(P, w, sc, mask_a, f, p.solve_chunks, p.solve_rows);
    a.g = g;
    a.g_eff_out = w.g_eff;
    a.log_b = w.log_b;
    a.mask_b = mask_b;
    a.rho_b = sc.rho_b;
    a.omr_b = sc.omr_b;
    a.bar = status_bar(w.status);
    const int64_t units = P.B * p.solve_chunks;
    if (p.cluster == 2) return launch_solve_cl<2>(a, units, s);
    if (p.cluster == 4) return launch_solve_cl<4>(a, units, s);
    if (p.cluster == 8) return launch_solve_cl<8>(a, units, s);
    return fail(SK_ERR_LAYOUT, "no single-read iteration for this M");
}

}  // namespace sk

using namespace sk;

extern "C" {

int sk_solver_solve(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb, int64_t sCn,
                    int64_t sCm, const uint8_t* mask_a, const uint8_t* mask_b, double epsilon,
                    double tau_a, double tau_b, float* f, float* g, void* workspace,
                    size_t workspace_bytes, void* stream) {
    clear_error();
    if (int e = check_problem(C, B, N, M, epsilon)) return e;
    if (!f || !g) return fail(SK_ERR_ARG, "f and g must be non-NULL");
    const SolveWs w = carve_solve(workspace, B, N, M);
    if (!workspace || workspace_bytes < w.bytes)
        return fail(SK_ERR_WORKSPACE, "workspace smaller than sk_forward_workspace_bytes");
    const Problem P{C, B, N, M, sCb, sCn, sCm};
    const SweepPlan p = make_plan(C, B, N, M, sCb, sCn, sCm);
    if (!p.persist)
        return fail(SK_ERR_LAYOUT, "this shape / layout has no persistent solve on this device");
    const Scalars sc = make_scalars(epsilon, tau_a, tau_b);
    return launch_fused_solve(P, p, w, sc, mask_a, mask_b, f, g, (cudaStream_t)stream);
}

}  // extern "C"
