// sk_internal.h -- host-side plumbing shared by the translation units of
// libsinkhorn_b200.so: error reporting, launch planning, workspace layout.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

#include "../../include/sinkhorn_b200.h"

namespace sk {

// The status region of a solve's workspace: the Status record (bytes 0-63),
// the persistent solve's grid-barrier counter (bytes 128-191), the
// row-sharded exchange's CTA counter (bytes 192-255), then the
// column finish's per-group arrival counters and per-group residuals:
// k_col_finish's CTAs arrive in groups of 32 (one counter and one residual
// word per group) and the last CTA of each group arrives at the Status
// ticket, so no counter sees more than 32 atomics per iteration.
// fin_groups() of each for B*M columns; all zero between launches.
constexpr int kFinGroupCtas = 32;
constexpr int64_t kFinColsPerCta = 64;
__host__ __device__ inline int64_t fin_groups(int64_t BM) {
    const int64_t ctas = (BM + kFinColsPerCta - 1) / kFinColsPerCta;
    return (ctas + kFinGroupCtas - 1) / kFinGroupCtas;
}
// The row-sharded exchange's CTA counter (sk_peer.cu) at byte 192.
__host__ __device__ inline unsigned* status_push_ticket(void* status) {
    return reinterpret_cast<unsigned*>(reinterpret_cast<char*>(status) + 192);
}
// Ranks of a row-sharded solve that exchange over peer memory.
constexpr int kMaxPeers = 8;
__host__ __device__ inline unsigned* status_fin_count(void* status) {
    return reinterpret_cast<unsigned*>(reinterpret_cast<char*>(status) + 256);
}
__host__ __device__ inline unsigned* status_fin_res(void* status, int64_t BM) {
    return status_fin_count(status) + fin_groups(BM);
}
// Bytes of the status region of a solve over B*M columns.
inline size_t status_bytes(int64_t BM) { return 256 + 2 * sizeof(unsigned) * fin_groups(BM); }

// thread-local last error (sk_last_error)
void set_error(const std::string& msg);
void clear_error();

int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

#define SK_CUDA(call)                                      \
    do {                                                   \
        cudaError_t e__ = (call);                          \
        if (e__ != cudaSuccess) return ::sk::cuda_fail(e__, #call); \
    } while (0)

#define SK_LAUNCHED(what)                                  \
    do {                                                   \
        cudaError_t e__ = cudaGetLastError();              \
        if (e__ != cudaSuccess) return ::sk::cuda_fail(e__, what); \
    } while (0)

// Launch a kernel as a programmatic dependent of the previous kernel on the
// stream (the kernel must start with pdl_wait(); see sk_common.cuh). Errors
// are reported by the caller's SK_LAUNCHED.
template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    (void)cudaLaunchKernelEx(&cfg, kernel, args...);
}

constexpr size_t kAlign = 256;
inline size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

// Shape of one sweep launch.
struct SweepPlan {
    int vec;            // 4: float4 fast path, 1: strided scalar path
    int tpr;            // row-sweep threads per row
    int64_t ntiles;     // column tiles of the column sweep
    int64_t nbands;     // row bands of the column sweep
    int64_t band_rows;  // rows per band (multiple of 64)
    int fused;          // 1: sk_forward runs the single-read iteration (sk_fused.cu)
    int fused_ok;       // 1: the shape / layout has a single-read iteration
    int col_tma;        // 1: column sweep fed by tensor-map copies (float4 layouts)
    int64_t chunks;     // fused: row chunks per batch item
    int64_t rows_per_chunk;
    int bf16;           // 1: C holds bf16 (the 4-wide kernels with bf16 loads)
    int fused_rows;     // 1: the single-read iteration is k_rows_fused (sk_fused_rows.cu),
                        // 2: k_row_warps (sk_row_warps.cu)
    int cluster;        // CTAs per cluster of the row-split single-read iteration (1, 2, 4, 8)
    int persist;        // 1: sk_forward may run the whole solve as one persistent launch
    int64_t solve_chunks;  // its row chunks per item (one wave of clusters)
    int64_t solve_rows;    // and rows per chunk
};

// Fused single-read iteration: whether a shape qualifies, and its chunking
// (whole waves of co-resident 2-CTA clusters). Defined in sk_fused.cu.
// single_cta = false keeps 2-CTA clusters for 2048 < M < 8192 (the bf16
// plan: its kernels exist for 2-CTA clusters only).
void plan_fused(SweepPlan& p, int64_t B, int64_t N, int64_t M, bool single_cta = true);
// Upper bound of the chunks per item plan_fused may choose (workspace sizing);
// 0 when the shape has no fused iteration.
int64_t fused_max_chunks(int64_t B, int64_t N, int64_t M);

// The single-read iteration for 512 <= M <= 2048 (sk_fused_rows.cu): shapes,
// chunks per item, and the chunk bound for workspace sizing.
bool rows_fused_shape(int64_t N, int64_t M);
int64_t rows_fused_chunks(int64_t B, int64_t N);
int64_t rows_fused_max_chunks(int64_t B, int64_t N);
// The single-read iteration with a warp per row for 512 < M <= 1024
// (sk_row_warps.cu): shapes, chunks per item and their bound.
bool row_warps_shape(int64_t N, int64_t M);
int64_t row_warps_chunks(int64_t B, int64_t N);
int64_t row_warps_max_chunks(int64_t B, int64_t N);

// Banding depends on (B,N,M) only, so workspace sizes are known before the
// strides are: column sweeps target ~4 waves of 8 CTAs per SM on 148 SMs.
int64_t col_bands(int64_t B, int64_t N, int64_t M, int64_t* band_rows);
// Tickets are sized for the scalar path (the larger tile count).
int64_t max_col_tiles(int64_t M);

SweepPlan make_plan(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                    int64_t sCn, int64_t sCm);
// The plan for a bf16 C (its address passed as `C`): the 4-wide layout only
// (vec = 0 in the result when C does not qualify), register column sweep, the
// fused iteration where M % 16 == 0 keeps half-rows 16-byte multiples.
SweepPlan make_plan_bf16(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                         int64_t sCn, int64_t sCm);

// Workspace carve-up of a solve (sk_forward and the iteration steps).
struct SolveWs {
    void* status;     // Status record
    float* log_a;     // (B,N)
    float* log_b;     // (B,M)
    float* f_eff;     // (B,N)
    float* g_eff;     // (B,M)
    int* ranges;      // (B,4)
    unsigned* tickets;
    float* partial;   // (B, nbands, M)
    float* fparts;    // fused path: (chunks, B*M + 1) column partials
    size_t bytes;
};
SolveWs carve_solve(void* base, int64_t B, int64_t N, int64_t M);

int check_problem(const float* C, int64_t B, int64_t N, int64_t M, double epsilon);

}  // namespace sk
