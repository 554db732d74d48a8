// sk_solve.cuh -- solve plumbing shared by the forward and backward units:
// the init kernel, sweep launches and the host iteration loop (sk_forward.cu).
#pragma once

#include "sk_internal.h"
#include "sk_sweep.cuh"

namespace sk {

struct Problem {
    const float* C;
    int64_t B, N, M, sCb, sCn, sCm;
};

struct Scalars {
    float k, eps, rho_a, omr_a, rho_b, omr_b;  // k = 1/eps
};

// rho = eps/(eps+tau), 0 for tau = inf (compute_rho, unbalanced.py:13-25)
Scalars make_scalars(double eps, double tau_a, double tau_b);

void launch_row(const SweepPlan& p, const RowArgs& ra, cudaStream_t s);
void launch_col(const SweepPlan& p, const ColArgs& ca, cudaStream_t s);

RowArgs make_row_args(const Problem& P, const SolveWs& w, const Scalars& sc,
                      const uint8_t* mask_a, float* f, const float* f_in);
ColArgs make_col_args(const Problem& P, const SweepPlan& p, const SolveWs& w,
                      const Scalars& sc, const uint8_t* mask_b, float* g,
                      const float* g_in);

// Device prologue: marginals, logs, potentials, effective potentials, ranges,
// tickets, status. keep = 1 keeps f/g as the starting point. iter_masks = 0
// lets masks shape the default marginals only (the iterations ignore them).
int init_solve(const Problem& P, const SolveWs& w, const float* a, const float* b,
               const uint8_t* mask_a, const uint8_t* mask_b, float* f, float* g,
               int max_iters, int check_every, float thr, int decide, int keep,
               cudaStream_t s, int iter_masks = 1);

// The whole solve in one launch when one item's C fits in an SM's shared
// memory (sk_onchip.cu); *ran = false when it does not qualify (the caller
// runs the two-sweep loop). check_every 0: no convergence checks.
int try_onchip_solve(const Problem& P, const SolveWs& w, const Scalars& sc,
                     const uint8_t* mask_a, const uint8_t* mask_b, float* f, float* g,
                     int max_iters, int check_every, float thr, cudaStream_t s, bool* ran);

// Enqueue up to max_iters iterations; with `checks`, poll the device decision
// one check period behind and stop enqueueing once done.
int run_solve(const Problem& P, const SweepPlan& p, const RowArgs& ra, const ColArgs& ca,
              int max_iters, int check_every, bool checks, cudaStream_t s, bool allow_poll,
              const SolveWs* fused_ws = nullptr, const Scalars* sc = nullptr);

int read_status(const void* st, Status* out, cudaStream_t s);

// Fused single-read f-update + column partials over the workspace's chunks
// (sk_fused.cu), and the merge / g-update / check of a partial set
// (sk_shard.cu): one fused iteration is launch_fused + launch_col_finish.
// A step's outputs beside the in-place default: the previous f from f_in and
// the new one into f_out (the backward's recompute keeps every iteration's),
// the rows' LSE (natural log) into lse_out, and whether the softmin takes the
// forward's isinf guard.
struct StepOut {
    const float* f_in;
    float* f_out;
    float* lse_out;
    int guard;
};
int launch_fused(const Problem& P, const SweepPlan& p, const SolveWs& w, const Scalars& sc,
                 const uint8_t* mask_a, float* f, cudaStream_t s, const StepOut* out = nullptr);
int launch_rows_fused(const Problem& P, const SweepPlan& p, const SolveWs& w,
                      const Scalars& sc, const uint8_t* mask_a, float* f, cudaStream_t s,
                      const StepOut* out = nullptr);
int launch_row_warps(const Problem& P, const SweepPlan& p, const SolveWs& w,
                      const Scalars& sc, const uint8_t* mask_a, float* f, cudaStream_t s,
                      const StepOut* out = nullptr);
// The whole solve as one cooperative launch (sk_fused_solve.cu) on a plan
// with `persist`: every unit resident, merge and decision between bounded
// grid barriers.
int launch_fused_solve(const Problem& P, const SweepPlan& p, const SolveWs& w,
                       const Scalars& sc, const uint8_t* mask_a, const uint8_t* mask_b,
                       float* f, float* g, cudaStream_t s);
// g_in (nullptr: g itself) is the previous g; lse_out (nullptr: none) gets
// the merged column LSEs (natural log); guard as StepOut's.
int launch_col_finish(const float* parts, int nparts, int64_t stride, int64_t B, int64_t M,
                      const uint8_t* mask_b, const float* log_b, float* g, float* g_eff,
                      const Scalars& sc, void* status, cudaStream_t s,
                      const float* g_in = nullptr, float* lse_out = nullptr, int guard = 1);
// The same finish over the P ranks' vectors of the peer exchange (sk_peer.cu):
// waits for the ranks' flags of this iteration, reads parity (iter & 1).
int launch_col_finish_peer(const float* parts, int nparts, int64_t stride, int64_t par_stride,
                           const unsigned* flags, int64_t B, int64_t M, const uint8_t* mask_b,
                           const float* log_b, float* g, float* g_eff, const Scalars& sc,
                           void* status, cudaStream_t s);


// One reverse step of the backward on the single read (sk_bwd_rows.cu): the
// row pass with gf^k and -lse_c^k, the row adjoint step (Fb, ff^k, -lse_r^k,
// dlog_a) and, with col_pass, the chunks' column sums S into parts.
struct BwdRowsStep {
    const float *fk, *gprev, *gf, *bc, *lr;
    const uint8_t *mask_a, *mask_b;  // full mode's masks, else nullptr
    float *Fb, *ff, *ar, *dlog_a;
    float* parts;
    int64_t pstride, chunks;
    float k2, eps, rho, omr;
    int full, col_pass;
    void* status;
};
bool bwd_rows_shape(const SweepPlan& p, int64_t N, int64_t M);
int64_t bwd_rows_chunks(int64_t B, int64_t N, int64_t M);
int launch_bwd_rows(const Problem& P, const BwdRowsStep& r, cudaStream_t s);

}  // namespace sk
