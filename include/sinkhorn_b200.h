/*
 * sinkhorn_b200.h -- C ABI of the B200 (sm_100a) log-domain Sinkhorn kernels.
 *
 * One shared library, libsinkhorn_b200.so, exports the functions below with
 * plain pointers and sizes. Every pointer argument named C, a, b, f, g, P,
 * mask_*, grad_*, d* and workspace is DEVICE memory on the current CUDA
 * device; scalar outputs (n_iters, converged, K) are HOST pointers.
 *
 * Layouts: C is (B,N,M) fp32 addressed as C[b*sCb + i*sCn + j*sCm] (strides
 * in elements, any sign-free layout; contiguous row-major is the fast path).
 * Row vectors (a, f, mask_a, ...) are dense (B,N), column vectors are dense
 * (B,M), masks are uint8 (nonzero = valid) and may be NULL ("all valid").
 * tau = +INFINITY means a balanced marginal (the reference's tau=None).
 *
 * Ownership: the caller allocates every device buffer, the workspace
 * included (sizes from the *_workspace_bytes queries). The library keeps no
 * device state between calls, with two documented exceptions: the built-in
 * scratch of sk_lse_col_noalloc, and -- host side -- the forward solves'
 * convergence polling, which keeps per calling thread and device 128 bytes of
 * pinned host memory and two CUDA events, created on first use and kept until
 * the process exits. All work is queued on `stream` (a cudaStream_t, NULL =
 * legacy default stream).
 *
 * Errors: every entry point returns SK_OK (0) or an sk_status code;
 * sk_last_error() returns a message for the calling thread's last failure.
 *
 * Each declaration names the reference interface it replaces (paths are
 * relative to the vv137/sinkhorn project).
 */
#ifndef SINKHORN_B200_H
#define SINKHORN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum sk_status {
    SK_OK = 0,
    SK_ERR_ARG = 1,        /* bad size, epsilon, iteration count, NULL pointer */
    SK_ERR_LAYOUT = 2,     /* unsupported strides / alignment                  */
    SK_ERR_WORKSPACE = 3,  /* workspace missing or too small                   */
    SK_ERR_CUDA = 4,       /* a CUDA runtime call or kernel launch failed      */
    SK_ERR_DEVICE = 5,     /* a kernel reported an error through its status    */
    SK_ERR_TIMEOUT = 6     /* a bounded device-side wait gave up               */
};

/* Library version, major*10000 + minor*100 + patch. */
int sk_version(void);

/* Message of the calling thread's most recent failure ("" if none). */
const char* sk_last_error(void);

/* ---------------------------------------------------------------------- */
/* Forward solve.                                                          */

/* Workspace bytes needed by sk_forward for a (B,N,M) problem. */
size_t sk_forward_workspace_bytes(int64_t B, int64_t N, int64_t M);

/*
 * Full Sinkhorn solve: f (B,N) and g (B,M) from zero potentials.
 * Replaces sinkhorn_forward_triton (src/sinkhorn/triton/forward.py:85-186),
 * the body of sinkhorn(backend="triton") (src/sinkhorn/sinkhorn.py:212-218).
 *
 * a, b: marginals or NULL (default: uniform 1/N, or mask/count when a mask is
 * given; forward.py:132-142). epsilon > 0. rho = eps/(eps+tau).
 * Convergence: every `check_every` iterations (10 = the Triton path,
 * 1 = the PyTorch path), stop when max over the whole batch of |f-f_prev| and
 * |g-g_prev| is below `threshold` (threshold <= 0: never, run max_iters).
 * Outputs f, g (device) and *n_iters, *converged (host).
 */
int sk_forward(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
               int64_t sCn, int64_t sCm, const float* a, const float* b,
               const uint8_t* mask_a, const uint8_t* mask_b, double epsilon,
               double tau_a, double tau_b, int max_iters, double threshold,
               int check_every, float* f, float* g, void* workspace,
               size_t workspace_bytes, int* n_iters, int* converged, void* stream);

/*
 * The same solve started from the potentials already in f and g (warm start,
 * checkpoint-resume, eps-annealing): the mechanism of _sinkhorn_iters_from_init
 * (src/sinkhorn/autograd.py:134-178) exposed on the forward path, with its
 * masks and convergence check. Resuming a threshold-0 solve from its (f, g)
 * after k iterations gives the potentials of one run of k + the new max_iters
 * iterations; n_iters counts the iterations of this call.
 */
int sk_forward_warm(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                    int64_t sCn, int64_t sCm, const float* a, const float* b,
                    const uint8_t* mask_a, const uint8_t* mask_b, double epsilon,
                    double tau_a, double tau_b, int max_iters, double threshold,
                    int check_every, float* f, float* g, void* workspace,
                    size_t workspace_bytes, int* n_iters, int* converged, void* stream);

/*
 * The same solve on a bf16 cost matrix (C: the 16-bit bf16 patterns, strides
 * in elements): every element is widened exactly to fp32 in the kernels and
 * the arithmetic is the fp32 path's, so the result is the fp32 solve of the
 * bf16-rounded costs while C's traffic is halved. Opt-in reduced-precision
 * input with no counterpart in the reference (whose Triton path loads C at its
 * own dtype, src/sinkhorn/triton/lse_kernel.py:73). Needs unit column stride,
 * 16-byte aligned rows and M % 4 == 0 (else SK_ERR_LAYOUT). Same workspace as
 * sk_forward.
 */
int sk_forward_bf16(const uint16_t* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                    int64_t sCn, int64_t sCm, const float* a, const float* b,
                    const uint8_t* mask_a, const uint8_t* mask_b, double epsilon,
                    double tau_a, double tau_b, int max_iters, double threshold,
                    int check_every, float* f, float* g, void* workspace,
                    size_t workspace_bytes, int* n_iters, int* converged, void* stream);

/* ---------------------------------------------------------------------- */
/* Step-level solve (for drivers that interleave their own work, e.g. a    */
/* collective, between sweeps). The workspace has the sk_forward layout    */
/* and starts with a 64-byte status record of int32 fields: iter (+0),     */
/* done (+4), n_iters (+8), converged (+12), residual (+16, float32: max   */
/* |delta| of the last check iteration), ticket (+20), max_iters (+24),    */
/* check_every (+28), threshold (+32, float32), decide (+36).              */
/* These steps break sinkhorn_forward_triton's loop                        */
/* (src/sinkhorn/triton/forward.py:161-184) into its pieces.              */

/*
 * Prologue of forward.py:119-156: default marginals, clamped logs, f = g = 0,
 * masks, status (iter 0). check_every = 0 disables residual checks;
 * decide = 1 takes the convergence decision on the device, decide = 0 leaves
 * the residual of each check iteration in the status for the caller.
 */
int sk_solver_init(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                   int64_t sCn, int64_t sCm, const float* a, const float* b,
                   const uint8_t* mask_a, const uint8_t* mask_b, int max_iters,
                   double threshold, int check_every, int decide, float* f, float* g,
                   void* workspace, size_t workspace_bytes, void* stream);

/* One f-update sweep (sinkhorn_row_update, forward.py:14-49, plus the row
 * masking of forward.py:168-169). */
int sk_solver_row_sweep(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                        int64_t sCn, int64_t sCm, const uint8_t* mask_a, double epsilon,
                        double tau_a, float* f, void* workspace, size_t workspace_bytes,
                        void* stream);

/* One g-update sweep (sinkhorn_col_update, forward.py:52-82, plus the column
 * masking and the iteration's check, forward.py:170-182). Advances iter. */
int sk_solver_col_sweep(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                        int64_t sCn, int64_t sCm, const uint8_t* mask_b, double epsilon,
                        double tau_b, float* g, void* workspace, size_t workspace_bytes,
                        void* stream);

/*
 * Row-sharded solve (C split by rows over P ranks; each rank calls these on
 * its rows (B, N_local, M) with a full copy of g). The column half-step of
 * forward.py:52-82 becomes: sk_solver_col_partial writes this rank's column
 * LSE over its rows into partial[0..B*M) (natural log) and its |delta f|
 * residual into partial[B*M]; the caller all-gathers the P vectors into
 * parts (P, B*M+1); sk_solver_col_finish merges them and applies the g
 * update, mask, residual, check and iteration counter -- identically on every
 * rank. N is the local row count (it selects the workspace layout); P <= 256.
 */
int sk_solver_col_partial(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                          int64_t sCn, int64_t sCm, double epsilon, float* partial,
                          void* workspace, size_t workspace_bytes, void* stream);

int sk_solver_col_finish(const float* parts, int P, int64_t B, int64_t N, int64_t M,
                         const uint8_t* mask_b, double epsilon, double tau_b, float* g,
                         void* workspace, size_t workspace_bytes, void* stream);

/*
 * The same column half-step on the single-read iteration (shapes with a
 * fused plan): after sk_solver_fused_step on the rank's rows,
 * sk_solver_chunk_merge writes the rank's column LSE over its rows into
 * out[0..B*M) and its f residual of a check iteration into out[B*M] (a NaN
 * as +inf), from the step's chunk partials. Then either all-gather and
 * sk_solver_col_finish as above, or the all-reduce merge: gmax = the
 * element-wise MAX over ranks of out (an all-reduce), sk_solver_rank_rescale
 * forms exp(out - gmax) into s, s is summed over ranks (an all-reduce) and
 * sk_solver_col_finish_pairs applies the g-update to the column LSEs
 * gmax + log(s), with gmax[B*M] as the ranks' f residual. Every rank takes
 * the same decision. Replace the column update of forward.py:52-82 (and the
 * batch-wide check of :176-182) when C is split by rows.
 */
int sk_solver_chunk_merge(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                          int64_t sCn, int64_t sCm, float* out, void* workspace,
                          size_t workspace_bytes, void* stream);
int sk_solver_rank_rescale(const float* local, const float* gmax, float* out, int64_t n,
                           void* stream);
int sk_solver_col_finish_pairs(const float* pair_m, const float* pair_s, int64_t B, int64_t N,
                               int64_t M, const uint8_t* mask_b, double epsilon, double tau_b,
                               float* g, void* workspace, size_t workspace_bytes,
                               void* stream);

/*
 * The same exchange over NVLink peer memory instead of a collective call
 * (ranks of one node, one GPU each, P <= 8). Each rank allocates one receive
 * buffer of sk_peer_buffer_bytes(P, B, M) bytes with sk_peer_buffer_alloc
 * (zeroed), exports it with sk_peer_handle (a 64-byte CUDA IPC handle), and
 * opens the others' with sk_peer_open; bases[q] is rank q's buffer as seen
 * by this process (its own pointer for q = rank). Before a solve's first
 * iteration every rank calls sk_peer_reset on its own buffer and the ranks
 * meet at a host barrier. Per iteration, after sk_solver_fused_step:
 * sk_solver_chunk_merge_peer stores the rank's column LSE vector (as
 * sk_solver_chunk_merge forms it) into slot [iteration parity][rank] of every
 * rank's buffer and then raises the rank's flag in each (release at system
 * scope); sk_solver_col_finish_peer waits, bounded, until all P flags of the
 * iteration are up (SK_ERR_TIMEOUT through the status otherwise), merges the
 * P vectors in rank order and applies the g-update, residual, check and
 * iteration counter, identically on every rank. No host synchronisation and
 * no collective call per iteration. After the last solve: a host barrier,
 * sk_peer_close on the opened buffers, sk_peer_buffer_free on the own one.
 * No reference counterpart (the reference runs on one device).
 */
size_t sk_peer_buffer_bytes(int P, int64_t B, int64_t M);
int sk_peer_buffer_alloc(size_t bytes, void** ptr);
int sk_peer_buffer_free(void* ptr);
int sk_peer_handle(const void* ptr, void* handle);
int sk_peer_open(const void* handle, void** ptr);
int sk_peer_close(void* ptr);
int sk_peer_reset(void* own, int P, int64_t B, int64_t M, void* stream);
int sk_solver_chunk_merge_peer(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                               int64_t sCn, int64_t sCm, const void* const* bases, int P,
                               int rank, void* workspace, size_t workspace_bytes, void* stream);
int sk_solver_col_finish_peer(const void* own, int P, int64_t B, int64_t N, int64_t M,
                              const uint8_t* mask_b, double epsilon, double tau_b, float* g,
                              void* workspace, size_t workspace_bytes, void* stream);

/*
 * Convergence decision of a solve whose kernels ran with decide = 0 after the
 * caller reduced the residual (workspace status, res_bits) across ranks --
 * the batch-sharded solve's global check (forward.py:176-182: the max over
 * the whole batch). Queued on the stream: no host synchronisation.
 */
int sk_solver_decide(void* workspace, void* stream);

/*
 * Single-read iteration (same loop as above, one pass over C instead of two):
 * sk_solver_fused_step updates f and forms per-chunk column partials while
 * each row is in shared memory; sk_solver_fused_finish merges the chunks and
 * applies the g update, residual, check and iteration counter. Only for the
 * shapes sk_plan_query reports as fused (contiguous 16-byte aligned rows, and
 * 512 <= M <= 2048 with M % 4 == 0, or 2048 < M <= 16384 with M % 8 == 0).
 * sk_forward runs this iteration itself when M >= 8192, and for
 * 512 <= M <= 2048 when the batch has at least 4736 rows (on B200 per
 * iteration: N=M=16384 0.185 ms against 0.446 ms for the two sweeps; B=16
 * N=M=2048 0.078 against 0.118 ms); elsewhere the two sweeps are faster and
 * these steps opt in.
 */
int sk_solver_fused_step(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                         int64_t sCn, int64_t sCm, const uint8_t* mask_a, double epsilon,
                         double tau_a, float* f, void* workspace, size_t workspace_bytes,
                         void* stream);

/*
 * The remaining iterations of a solve set up by sk_solver_init (decide = 1)
 * as one persistent launch of the single-read iteration: every unit of the
 * problem on its own co-resident cluster, the chunk merge, g-update and
 * convergence decision between bounded grid barriers, the ring refilled with
 * the next iteration's rows meanwhile. Results are bit-identical to the loop
 * of sk_solver_fused_step + sk_solver_fused_finish. For the shapes
 * sk_plan_query reports with fused = 3 (SK_ERR_LAYOUT otherwise, or an
 * SK_ERR_CUDA launch error where the device refuses a cooperative cluster
 * launch). An opt-in alternative: sk_forward runs the loop, which measured as
 * fast or faster on B200 (N=M=16384: 0.185 ms per iteration for the loop,
 * 0.219 ms for this launch; within 5% either way at N=M=8192 and 12288).
 * Replaces the loop of sinkhorn_forward_triton
 * (src/sinkhorn/triton/forward.py:161-184).
 */
int sk_solver_solve(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb, int64_t sCn,
                    int64_t sCm, const uint8_t* mask_a, const uint8_t* mask_b, double epsilon,
                    double tau_a, double tau_b, float* f, float* g, void* workspace,
                    size_t workspace_bytes, void* stream);

int sk_solver_fused_finish(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                           int64_t sCn, int64_t sCm, const uint8_t* mask_b, double epsilon,
                           double tau_b, float* g, void* workspace, size_t workspace_bytes,
                           void* stream);

/* Which kernels a problem of this shape/layout runs on (host outputs; NULL
 * allowed): vec = 4 for the float4 path, 1 for the strided one; fused = 0 when
 * the shape has no single-read iteration, 1 when it has one (opt-in steps), 2
 * when sk_forward runs it, 3 when sk_forward runs it and sk_solver_solve is
 * available too; chunks = row chunks per item of the fused path.
 * A diagnostic with no reference counterpart. */
int sk_plan_query(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb, int64_t sCn,
                  int64_t sCm, int* vec, int* fused, int64_t* chunks);

/* Diagnostic with no reference counterpart: the device's ex2.approx.f32
 * throughput (results per second, all SMs busy), the exponential floor of a
 * sweep's roofline. scratch: device buffer of sk_probe_ex2_scratch_bytes()
 * (one float per probe thread); synchronizes the stream. */
size_t sk_probe_ex2_scratch_bytes(void);
int sk_probe_ex2_rate(float* scratch, size_t scratch_bytes, double* ex2_per_second,
                      void* stream);

/* Diagnostic (no reference counterpart): one bounded wait of the kind the
 * pipelined kernels use -- kind 0 a local mbarrier, 1 a cluster peer's
 * st.async into this CTA's mbarrier, 2 a grid barrier of a cooperative
 * launch -- with at most `polls` polls, against a partner that arrives
 * (partner != 0: returns SK_OK) or never arrives (partner == 0: the wait
 * gives up, the kernel returns, and the call returns SK_ERR_TIMEOUT with the
 * context still usable). scratch: device buffer of
 * sk_probe_wait_scratch_bytes(); synchronizes the stream. */
size_t sk_probe_wait_scratch_bytes(void);
int sk_probe_wait_timeout(int kind, int partner, unsigned polls, void* scratch,
                          size_t scratch_bytes, void* stream);

/* Synchronous read of the status record (host outputs; any may be NULL). */
int sk_solver_status(const void* workspace, int* iter, int* done, int* n_iters,
                     int* converged, float* residual, void* stream);

/* ---------------------------------------------------------------------- */
/* Streaming softmins.                                                     */

/*
 * out[b,n] = -eps * logsumexp_m((g[b,m] - C[b,n,m]) / eps), 0 for a row with
 * no finite term. Replaces lse_row (src/sinkhorn/triton/lse_kernel.py:210-250).
 */
int sk_lse_row(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
               int64_t sCn, int64_t sCm, const float* g, double epsilon,
               float* out, void* stream);

/* Workspace bytes needed by sk_lse_col. */
size_t sk_lse_col_workspace_bytes(int64_t B, int64_t N, int64_t M);

/*
 * out[b,m] = -eps * logsumexp_n((f[b,n] - C[b,n,m]) / eps), 0 for an empty
 * column. Replaces lse_col (src/sinkhorn/triton/lse_kernel.py:253-293).
 */
int sk_lse_col(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
               int64_t sCn, int64_t sCm, const float* f, double epsilon,
               float* out, void* workspace, size_t workspace_bytes, void* stream);

/*
 * sk_lse_col for callers that cannot allocate device memory when they call
 * in -- a host application whose memory manager already holds the GPU's
 * memory, a service that forbids cudaMalloc on its request path (it can block
 * and synchronise the device), a binding without a device allocator. Same
 * result as sk_lse_col, but the scratch comes from an 8 MiB array built into
 * the library (kept on every GPU that loads it until the process exits), so
 * there is no workspace argument and nothing is allocated.
 * Limit: the scratch sk_lse_col_workspace_bytes(B,N,M) reports must fit in
 * 8 MiB -- roughly B*M below 2^21 columns in all (B=1 up to M of about two
 * million, B=32 below M=65536, B=64 at M=1024 needs 2 MiB); larger problems
 * get SK_ERR_WORKSPACE before any launch. All calls on a device share the
 * array: calls that overlap on the GPU race, so order them. The first call on
 * each device looks up the array's address and caches it; make it before any
 * stream capture, and do not call this entry point again on a device after
 * cudaDeviceReset in the same process (the cached address is then stale).
 * No counterpart in the reference: it exists only for callers that cannot
 * allocate.
 */
int sk_lse_col_noalloc(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                       int64_t sCn, int64_t sCm, const float* f, double epsilon,
                       float* out, void* stream);

/* ---------------------------------------------------------------------- */
/* Transport plan, cost, JVP.                                              */

/*
 * P[b,i,j] = exp((f[b,i] + g[b,j] - C[b,i,j]) / eps), 0 at masked rows and
 * columns; P is dense (B,N,M). Replaces SinkhornOutput.transport_plan
 * (src/sinkhorn/sinkhorn.py:27-54).
 */
int sk_transport_plan(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                      int64_t sCn, int64_t sCm, const float* f, const float* g,
                      double epsilon, const uint8_t* mask_a, const uint8_t* mask_b,
                      float* P, void* stream);

/* Workspace bytes needed by sk_marginal_error. */
size_t sk_marginal_error_workspace_bytes(int64_t B, int64_t N, int64_t M);

/*
 * out[0] = max over the whole batch of |sum_j P_ij - a_i| (0 at masked rows)
 * and |sum_i P_ij - b_j| (0 at masked columns), with P the masked plan of
 * sk_transport_plan, from one pass over C (P never stored); out is a device
 * float. Replaces compute_marginal_error (src/sinkhorn/pytorch/balanced.py:
 * 183-213).
 */
int sk_marginal_error(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                      int64_t sCn, int64_t sCm, const float* f, const float* g, const float* a,
                      const float* b, double epsilon, const uint8_t* mask_a,
                      const uint8_t* mask_b, float* out, void* workspace,
                      size_t workspace_bytes, void* stream);

/* ---- implicit-differentiation adjoint (src/sinkhorn/pytorch/implicit_diff.py) ----
 * Every entry below takes the plan either P-free, as (C, strides, f, g,
 * epsilon, mask_a, mask_b) with P = exp((f + g - C)/eps) recomputed tile by
 * tile and 0 at masked rows / columns, or as a dense contiguous plan P
 * (B,N,M) when P is non-NULL (C, f, g and the masks of the plan are then
 * ignored; C may be NULL).
 */

/* Workspace bytes needed by sk_plan_matvec. */
size_t sk_plan_matvec_workspace_bytes(int64_t B, int64_t N, int64_t M);

/*
 * Products with the plan from one pass: Px = P x (B,N) for x (B,M), Pty =
 * P^T y (B,M) for y (B,N), P1 = row sums (B,N), Pt1 = column sums (B,M); any
 * output may be NULL (an output needs its input). The plan contact of
 * schur_complement_matvec (implicit_diff.py:82-95).
 */
int sk_plan_matvec(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb, int64_t sCn,
                   int64_t sCm, const float* f, const float* g, double epsilon,
                   const uint8_t* mask_a, const uint8_t* mask_b, const float* P,
                   const float* x, const float* y, float* Px, float* Pty, float* P1,
                   float* Pt1, void* workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes needed by sk_implicit_matvec and sk_implicit_cg. */
size_t sk_implicit_workspace_bytes(int64_t B, int64_t N, int64_t M);

/*
 * One Jacobian product at the fixed point, r / c the plan's row / column sums
 * clamped at 1e-30 (two passes over the plan):
 *   mode 0: out = (1 + reg) v - J_T^T v   schur_complement_matvec, implicit_diff.py:45-104
 *   mode 1: out = J_T^T v                 vjp_sinkhorn,            implicit_diff.py:281-309
 *   mode 2: out = J_T v                   jvp_sinkhorn,            implicit_diff.py:253-278
 * with (J_T^T v)_f = rho_a v_f + (1 - rho_b) P (v_g / c),
 *      (J_T^T v)_g = rho_b v_g + (1 - rho_a) P^T (v_f / r),
 *      (J_T v)_f   = rho_a v_f + (1 - rho_a) (P v_g) / r,
 *      (J_T v)_g   = rho_b v_g + (1 - rho_b) (P^T v_f) / c.
 * Modes 1 and 2 write 0 at masked rows / columns.
 */
int sk_implicit_matvec(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                       int64_t sCn, int64_t sCm, const float* f, const float* g, double epsilon,
                       const uint8_t* mask_a, const uint8_t* mask_b, const float* P,
                       const float* v_f, const float* v_g, double rho_a, double rho_b,
                       double reg, int mode, float* out_f, float* out_g, void* workspace,
                       size_t workspace_bytes, void* stream);

/*
 * Batched conjugate gradients on (I - J_T^T + reg I) lambda = (rhs_f, rhs_g)
 * (cg_solve, implicit_diff.py:107-193): x0 = 0, at most max_iters iterations,
 * stopping after the first whose max over the batch of |r_b| is below
 * tol * max_b |rhs_b|. One pass over the plan per iteration; the stopping test
 * runs on the device, so nothing synchronises until the end. Writes lambda_f
 * (B,N), lambda_g (B,M) and, when non-NULL, grad_a = epsilon * lambda_f and
 * grad_b = epsilon * lambda_g (implicit_diff.py:246-247). *n_iters (host,
 * may be NULL; when given the call synchronises the stream) = iterations taken.
 */
int sk_implicit_cg(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb, int64_t sCn,
                   int64_t sCm, const float* f, const float* g, double epsilon,
                   const uint8_t* mask_a, const uint8_t* mask_b, const float* P,
                   const float* rhs_f, const float* rhs_g, double rho_a, double rho_b,
                   int max_iters, double tol, double reg, float* lambda_f, float* lambda_g,
                   float* grad_a, float* grad_b, void* workspace, size_t workspace_bytes,
                   int* n_iters, void* stream);

/*
 * dC = -(1/eps) P (lambda_f[:, None] + lambda_g[None, :]), 0 at masked rows /
 * columns, dense contiguous (B,N,M); P recomputed from C, f, g. The cost
 * gradient of implicit_gradient (implicit_diff.py:241-243).
 */
int sk_implicit_dC(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb, int64_t sCn,
                   int64_t sCm, const float* f, const float* g, double epsilon,
                   const uint8_t* mask_a, const uint8_t* mask_b, const float* lambda_f,
                   const float* lambda_g, float* dC, void* stream);

/* Workspace bytes needed by sk_cost. */
size_t sk_cost_workspace_bytes(int64_t B, int64_t N, int64_t M);

/*
 * out[b] = sum_ij P_ij C_ij with the unmasked plan, without materialising P.
 * Replaces SinkhornOutput.cost (src/sinkhorn/sinkhorn.py:56-67).
 */
int sk_cost(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb, int64_t sCn,
            int64_t sCm, const float* f, const float* g, double epsilon, float* out,
            void* workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes needed by sk_jvp / sk_jvp_plan. */
size_t sk_jvp_workspace_bytes(int64_t B, int64_t N, int64_t M);

/*
 * out_f = rho_a v_f + (1-rho_a) (P v_g)/(P 1), out_g likewise with P^T, where
 * P = exp((f+g-C)/eps) is recomputed tile by tile (never materialised);
 * the rho mix is skipped when rho == 0 and row/column sums are clamped at
 * 1e-38. P-free form of jvp_triton (src/sinkhorn/triton/jvp_kernel.py:113-182).
 */
int sk_jvp(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb, int64_t sCn,
           int64_t sCm, const float* f, const float* g, double epsilon,
           const float* v_f, const float* v_g, double rho_a, double rho_b,
           float* out_f, float* out_g, void* workspace, size_t workspace_bytes,
           void* stream);

/* Same on a materialised plan P (dense (B,N,M)): jvp_triton itself
 * (src/sinkhorn/triton/jvp_kernel.py:113-182). */
int sk_jvp_plan(const float* P, int64_t B, int64_t N, int64_t M, const float* v_f,
                const float* v_g, double rho_a, double rho_b, float* out_f,
                float* out_g, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Adjoint of the plan for an upstream gradient grad_P (dense (B,N,M)):
 * W = grad_P * P / eps; dC = -W (0 where masked), df = sum_j W, dg = sum_i W.
 * Any of dC/df/dg may be NULL. Backward of transport_plan as autograd
 * differentiates src/sinkhorn/sinkhorn.py:47-54.
 */
int sk_plan_backward(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                     int64_t sCn, int64_t sCm, const float* f, const float* g,
                     double epsilon, const uint8_t* mask_a, const uint8_t* mask_b,
                     const float* grad_P, float* dC, float* df, float* dg,
                     void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------- */
/* Backward.                                                               */

/* Workspace bytes needed by sk_backward with at most K recorded iterations
 * (K = grad_iters in truncated mode, max_iters in full mode). */
size_t sk_backward_workspace_bytes(int64_t B, int64_t N, int64_t M, int64_t K);

/*
 * Gradient of L = <f, grad_f> + <g, grad_g> with respect to C, log a, log b.
 * Replaces SinkhornFunction.backward (src/sinkhorn/autograd.py:61-131).
 * Truncated mode when 0 < grad_iters < max_iters: grad_iters iterations from
 * (f_star, g_star) on raw C, masks applied to the final potentials only
 * (autograd.py:83-97,134-178). Otherwise full mode: a fresh masked solve
 * from zeros with a per-iteration convergence check (autograd.py:98-113).
 * Outputs dC (dense (B,N,M)), dlog_a (B,N), dlog_b (B,M) (either may be
 * NULL) and *K (host): the number of iterations differentiated.
 */
int sk_backward(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                int64_t sCn, int64_t sCm, const float* a, const float* b,
                const uint8_t* mask_a, const uint8_t* mask_b, double epsilon,
                double tau_a, double tau_b, int max_iters, double threshold,
                int grad_iters, const float* f_star, const float* g_star,
                const float* grad_f, const float* grad_g, float* dC, float* dlog_a,
                float* dlog_b, void* workspace, size_t workspace_bytes, int* K,
                void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SINKHORN_B200_H */
