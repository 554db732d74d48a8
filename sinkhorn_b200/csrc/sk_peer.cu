// sk_peer.cu -- the row-sharded solve's per-iteration exchange over NVLink
// peer memory, without a collective library call.
//
// Every rank owns one receive buffer (sk_peer_buffer_alloc: a plain device
// allocation, shared with the other ranks of the node through a CUDA IPC
// handle), laid out as
//   vectors [2][P][stride] floats   (parity of the iteration, sending rank)
//   flags   [P] uint32              (per sending rank: the last iteration
//                                    number + 1 whose vector has landed)
// One iteration of the row-sharded solve on rank r is
//   sk_solver_fused_step        (its rows: f-update, chunk partials)
//   sk_solver_chunk_merge_peer  (its column LSE vector, B*M + 1 floats, is
//                                stored straight into slot [parity][r] of
//                                every rank's buffer, then, once every CTA's
//                                stores are fenced at system scope, the last
//                                CTA raises flag r in every rank's buffer
//                                with a release store)
//   sk_solver_col_finish_peer   (waits, bounded, for all P flags of this
//                                iteration with acquire loads, then merges
//                                the P vectors from its own buffer in rank
//                                order and applies the g-update, residual
//                                and check: identical on every rank)
// so the exchange costs one pass of stores over NVLink and no kernel launch
// or host synchronisation of its own. Two parities suffice: a rank writes
// slot [q] of iteration it + 2 only after it has passed the finish of
// iteration it + 1, which needed every rank's vector of it + 1, which each
// rank pushed after its own finish of iteration it had consumed slot [q].
// Each rank's kernels run on its own GPU; a waiting finish never waits for
// a kernel of its own GPU. No load here is a multicast.
#include <algorithm>
#include <cmath>
#include <cstring>

#include "sk_grid.cuh"
#include "sk_internal.h"
#include "sk_merge.cuh"
#include "sk_solve.cuh"

namespace sk {

static int64_t peer_stride(int64_t B, int64_t M) { return B * M + 4; }

static size_t peer_flags_offset(int P, int64_t B, int64_t M) {
    return align_up(sizeof(float) * 2 * (size_t)P * (size_t)peer_stride(B, M));
}

size_t peer_buffer_bytes(int P, int64_t B, int64_t M) {
    return peer_flags_offset(P, B, M) + align_up(sizeof(unsigned) * (size_t)P);
}

struct PeerPushArgs {
    const float* parts;  // this rank's chunk partials
    int nchunks;
    int64_t pstride, BM;
    float* dst[kMaxPeers];      // slot [0][rank] of every rank's buffer
    unsigned* flag[kMaxPeers];  // flag [rank] of every rank's buffer
    int P;
    int64_t par_stride;         // floats between the two parities: P * stride
    const Status* st;
    unsigned* ticket;           // this rank's CTA counter (status region), zero between launches
};

// The rank's column LSE vector (as k_chunk_merge forms it: the chunk
// partials merged in the fixed order of sk_merge.cuh, -inf for no term, and
// the rank's f residual of a check iteration in slot B*M, NaN as +inf),
// stored into every rank's buffer, then the flags.
__global__ void __launch_bounds__(256) k_chunk_merge_push(PeerPushArgs a) {
    pdl_trigger();
    __shared__ float2 sh_pair[2][kMergeSubsets][32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int cg = w / kMergeSubsets, sub = w % kMergeSubsets;
    const int64_t col = (int64_t)blockIdx.x * 64 + cg * 32 + lane;
    pdl_wait();
    const Status* st = a.st;
    if (read_volatile(&st->done)) return;  // the same on every rank and in every CTA
    const int iter = read_volatile(&st->iter);
    const int64_t off = (int64_t)(iter & 1) * a.par_stride;
    sh_pair[cg][sub][lane] = merge_subset<false>(a.parts + col, a.pstride, a.nchunks, sub,
                                                 col < a.BM);
    __syncthreads();
    if (sub == 0 && col < a.BM) {
        const float2 sp[kMergeSubsets] = {sh_pair[cg][0][lane], sh_pair[cg][1][lane],
                                          sh_pair[cg][2][lane], sh_pair[cg][3][lane]};
        float mm, ss;
        merge_subsets(mm, ss, sp);
        const float v = lse_of(mm, ss);
        for (int p = 0; p < a.P; ++p) a.dst[p][off + col] = v;
        __threadfence_system();  // this thread's stores before the CTA's arrival
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        float r = 0.f;
        if (is_check_iter(st, iter)) r = __uint_as_float(read_volatile((const int*)&st->res_bits));
        const float v = isnan(r) ? INFINITY : r;
        for (int p = 0; p < a.P; ++p) a.dst[p][off + a.BM] = v;
        __threadfence_system();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (atomicAdd(a.ticket, 1u) == gridDim.x - 1) {
            *a.ticket = 0u;
            __threadfence_system();
            for (int p = 0; p < a.P; ++p) st_release_sys(a.flag[p], (unsigned)iter + 1u);
        }
    }
}

__global__ void k_peer_reset(unsigned* flags, int P) {
    if (threadIdx.x < P) flags[threadIdx.x] = 0u;
}

}  // namespace sk

using namespace sk;

extern "C" {

size_t sk_peer_buffer_bytes(int P, int64_t B, int64_t M) {
    if (P < 1 || P > kMaxPeers || B <= 0 || M <= 0) return 0;
    return peer_buffer_bytes(P, B, M);
}

int sk_peer_buffer_alloc(size_t bytes, void** ptr) {
    if (!ptr || bytes == 0) return fail(SK_ERR_ARG, "ptr must be non-NULL and bytes positive");
    *ptr = nullptr;
    void* p = nullptr;
    SK_CUDA(cudaMalloc(&p, bytes));
    if (cudaMemset(p, 0, bytes) != cudaSuccess) {
        cudaFree(p);
        return fail(SK_ERR_CUDA, "cudaMemset of the peer buffer failed");
    }
    *ptr = p;
    return SK_OK;
}

int sk_peer_buffer_free(void* ptr) {
    if (ptr) SK_CUDA(cudaFree(ptr));
    return SK_OK;
}

int sk_peer_handle(const void* ptr, void* handle) {
    if (!ptr || !handle) return fail(SK_ERR_ARG, "NULL argument");
    cudaIpcMemHandle_t h;
    SK_CUDA(cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)));
    memcpy(handle, &h, sizeof(h));
    return SK_OK;
}

int sk_peer_open(const void* handle, void** ptr) {
    if (!handle || !ptr) return fail(SK_ERR_ARG, "NULL argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    *ptr = nullptr;
    SK_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return SK_OK;
}

int sk_peer_close(void* ptr) {
    if (ptr) SK_CUDA(cudaIpcCloseMemHandle(ptr));
    return SK_OK;
}

int sk_peer_reset(void* own, int P, int64_t B, int64_t M, void* stream) {
    if (!own || P < 1 || P > kMaxPeers || B <= 0 || M <= 0) return fail(SK_ERR_ARG, "bad argument");
    unsigned* flags = (unsigned*)((char*)own + peer_flags_offset(P, B, M));
    k_peer_reset<<<1, 32, 0, (cudaStream_t)stream>>>(flags, P);
    SK_LAUNCHED("k_peer_reset launch");
    return SK_OK;
}

int sk_solver_chunk_merge_peer(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                               int64_t sCn, int64_t sCm, const void* const* bases, int P,
                               int rank, void* workspace, size_t workspace_bytes,
                               void* stream) {
    if (int e = check_problem(C, B, N, M, 1.0)) return e;
    if (!bases || P < 1 || P > kMaxPeers || rank < 0 || rank >= P)
        return fail(SK_ERR_ARG, "bases must hold P (1..8) buffers and 0 <= rank < P");
    for (int p = 0; p < P; ++p)
        if (!bases[p]) return fail(SK_ERR_ARG, "a peer buffer is NULL");
    const SolveWs w = carve_solve(workspace, B, N, M);
    if (!workspace || workspace_bytes < w.bytes)
        return fail(SK_ERR_WORKSPACE, "workspace smaller than sk_forward_workspace_bytes");
    const SweepPlan p = make_plan(C, B, N, M, sCb, sCn, sCm);
    if (!p.fused_ok) return fail(SK_ERR_LAYOUT, "this shape / layout has no fused iteration");
    PeerPushArgs a{};
    a.parts = w.fparts;
    a.nchunks = (int)p.chunks;
    a.pstride = B * M + 4;
    a.BM = B * M;
    a.P = P;
    a.par_stride = (int64_t)P * peer_stride(B, M);
    for (int q = 0; q < P; ++q) {
        char* base = (char*)bases[q];
        a.dst[q] = (float*)base + (int64_t)rank * peer_stride(B, M);
        a.flag[q] = (unsigned*)(base + peer_flags_offset(P, B, M)) + rank;
    }
    a.st = (const Status*)w.status;
    a.ticket = status_push_ticket(w.status);
    launch_pdl(k_chunk_merge_push, dim3((unsigned)((B * M + 63) / 64)), dim3(256), 0,
               (cudaStream_t)stream, a);
    SK_LAUNCHED("k_chunk_merge_push launch");
    return SK_OK;
}

int sk_solver_col_finish_peer(const void* own, int P, int64_t B, int64_t N, int64_t M,
                              const uint8_t* mask_b, double epsilon, double tau_b, float* g,
                              void* workspace, size_t workspace_bytes, void* stream) {
    if (!own || !g) return fail(SK_ERR_ARG, "own and g must be non-NULL");
    if (P < 1 || P > kMaxPeers || B <= 0 || N <= 0 || M <= 0)
        return fail(SK_ERR_ARG, "bad P (1..8), B, N or M");
    if (!(epsilon > 0.0)) return fail(SK_ERR_ARG, "epsilon must be positive");
    const SolveWs w = carve_solve(workspace, B, N, M);
    if (!workspace || workspace_bytes < w.bytes)
        return fail(SK_ERR_WORKSPACE, "workspace smaller than sk_forward_workspace_bytes");
    const Scalars sc = make_scalars(epsilon, INFINITY, tau_b);
    const unsigned* flags = (const unsigned*)((const char*)own + peer_flags_offset(P, B, M));
    return launch_col_finish_peer((const float*)own, P, peer_stride(B, M),
                                  (int64_t)P * peer_stride(B, M), flags, B, M, mask_b, w.log_b,
                                  g, w.g_eff, sc, w.status, (cudaStream_t)stream);
}

}  // extern "C"
