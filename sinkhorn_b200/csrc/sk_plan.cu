// sk_plan.cu -- transport plan, cost, JVP and the plan adjoint (C ABI).
//
// The plan is one read of C and one write of P; the cost, the JVP and the
// plan adjoint never materialise P: they recompute exp((f+g-C)/eps) tile by
// tile inside the band kernel (sk_band.cuh).
#include <algorithm>
#include <cmath>

#include "sk_band.cuh"
#include "sk_internal.h"

namespace sk {

// ---------------------------------------------------------------------------
// P = exp(((f + g) - C)/eps), 0 at masked rows/columns (sinkhorn.py:47-54).
struct PlanArgs {
    const float* C;
    int64_t sCb, sCn, sCm;
    int64_t B, N, M;
    const float* f;
    const float* g;
    const uint8_t* mask_a;
    const uint8_t* mask_b;
    float inv_eps;
    float* P;
    int64_t nchunks;  // column chunks per row
};

constexpr int kPlanThreads = 256;

template <int VEC>
__global__ void __launch_bounds__(kPlanThreads) k_plan(PlanArgs a) {
    const int64_t cta = blockIdx.x;
    const int64_t row = cta / a.nchunks;
    const int64_t chunk = cta % a.nchunks;
    const int64_t b = row / a.N, i = row - b * a.N;
    const bool rvalid = a.mask_a == nullptr || a.mask_a[row] != 0;
    const float fi = a.f[row];
    const float* Crow = a.C + b * a.sCb + i * a.sCn;
    float* Prow = a.P + row * a.M;
    const float* gb = a.g + b * a.M;
    const uint8_t* mb = a.mask_b ? a.mask_b + b * a.M : nullptr;
    const int64_t j = (chunk * kPlanThreads + threadIdx.x) * VEC;
    if (j >= a.M) return;
    if constexpr (VEC == 4) {
        float4 out = make_float4(0.f, 0.f, 0.f, 0.f);
        if (rvalid) {
            const float4 c = ld_stream4(Crow + j);
            const float4 g = ld_vec4(gb + j);
            out.x = ex2(((fi + g.x) - c.x) * a.inv_eps * kLog2e);
            out.y = ex2(((fi + g.y) - c.y) * a.inv_eps * kLog2e);
            out.z = ex2(((fi + g.z) - c.z) * a.inv_eps * kLog2e);
            out.w = ex2(((fi + g.w) - c.w) * a.inv_eps * kLog2e);
            if (mb) {
                const uchar4 mm = *reinterpret_cast<const uchar4*>(mb + j);
                if (!mm.x) out.x = 0.f;
                if (!mm.y) out.y = 0.f;
                if (!mm.z) out.z = 0.f;
                if (!mm.w) out.w = 0.f;
            }
        }
        __stcs(reinterpret_cast<float4*>(Prow + j), out);
    } else {
        float out = 0.f;
        if (rvalid && (mb == nullptr || mb[j])) {
            const float c = ld_stream1(Crow + j * a.sCm);
            out = ex2(((fi + gb[j]) - c) * a.inv_eps * kLog2e);
        }
        Prow[j] = out;
    }
}

// Per-batch sum of a (B,N) vector in double, one CTA per batch item.
__global__ void k_batch_sum(const float* x, int64_t N, float* out) {
    __shared__ double sh[32];
    const int64_t b = blockIdx.x;
    double acc = 0.0;
    for (int64_t t = threadIdx.x; t < N; t += blockDim.x) acc += (double)x[b * N + t];
    acc = warp_sum_d(acc);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = 0.0;
        for (int q = 0; q < (int)(blockDim.x >> 5); ++q) s += sh[q];
        out[b] = (float)s;
    }
}

// max over the batch of |row_sum - a| (0 at masked rows) and |col_sum - b|
// (0 at masked columns); out[0] starts at 0 and takes an atomic max on the
// bit pattern of the non-negative errors (a NaN ranks above +inf, so it wins,
// as in torch.max).
__global__ void k_marginal_err(const float* rows, const float* cols, const float* a,
                               const float* b, const uint8_t* mask_a, const uint8_t* mask_b,
                               int64_t nr, int64_t nc, float* out) {
    __shared__ float sh[8];
    float e = 0.f;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < nr + nc;
         t += (int64_t)gridDim.x * blockDim.x) {
        float d;
        if (t < nr) {
            d = (mask_a && !mask_a[t]) ? 0.f : fabsf(rows[t] - a[t]);
        } else {
            const int64_t u = t - nr;
            d = (mask_b && !mask_b[u]) ? 0.f : fabsf(cols[u] - b[u]);
        }
        e = (d > e || isnan(d)) ? d : e;
    }
    float r = warp_max(e);
    if (__any_sync(0xffffffffu, isnan(e))) r = NAN;
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = r;
    __syncthreads();
    if (threadIdx.x == 0) {
        float rr = sh[0];
        for (int q = 1; q < (int)(blockDim.x >> 5); ++q)
            rr = (sh[q] > rr || isnan(sh[q])) ? sh[q] : rr;
        atomicMax(reinterpret_cast<unsigned*>(out), __float_as_uint(rr));
    }
}

// The JVP from finished sums (jvp_kernel.py:113-182 semantics):
// out = rho v + (1 - rho) s0 / max(s1, tiny), the mix skipped when rho = 0.
__global__ void k_jvp_tail(const float* s0, const float* s1, const float* v, int64_t n,
                           float rho, float omr, float* out) {
    for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n;
         k += (int64_t)gridDim.x * blockDim.x) {
        float r = s0[k] / fmaxf(s1[k], kTiny);
        if (rho != 0.f) r = rho * v[k] + omr * r;
        out[k] = r;
    }
}

// ---------------------------------------------------------------------------
// Band pass plumbing

struct BandWs {
    float* row_part;
    float* col_part;
    unsigned* tick_row;
    unsigned* tick_col;
    size_t tick_bytes;
    size_t bytes;
};

static BandWs carve_band(void* base, int64_t B, int64_t N, int64_t M) {
    int64_t br;
    const int64_t nb = col_bands(B, N, M, &br);
    const int64_t nt = max_col_tiles(M);  // scalar-path upper bound
    BandWs w{};
    char* p = (char*)base;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        char* r = p ? p + off : nullptr;
        off += align_up(bytes);
        return r;
    };
    // tickets first, contiguous, so one memset clears them
    w.tick_bytes = sizeof(unsigned) * B * (nb + nt);
    w.tick_row = (unsigned*)take(w.tick_bytes);
    w.tick_col = w.tick_row ? w.tick_row + B * nb : nullptr;
    w.row_part = (float*)take(sizeof(float) * 2 * B * N * nt);
    w.col_part = (float*)take(sizeof(float) * 2 * B * nb * M);
    w.bytes = off;
    return w;
}

size_t band_workspace_bytes(int64_t B, int64_t N, int64_t M) {
    return carve_band(nullptr, B, N, M).bytes;
}

int launch_band(BandArgs a, bool vec4, void* ws, cudaStream_t s) {
    const BandWs w = carve_band(ws, a.B, a.N, a.M);
    a.nbands = col_bands(a.B, a.N, a.M, &a.band_rows);
    a.ntiles = (a.M + 32 * (vec4 ? 4 : 1) - 1) / (32 * (vec4 ? 4 : 1));
    a.row_part = w.row_part;
    a.col_part = w.col_part;
    a.tick_row = w.tick_row;
    a.tick_col = w.tick_col;
    SK_CUDA(cudaMemsetAsync(w.tick_row, 0, w.tick_bytes, s));
    const unsigned grid = (unsigned)(a.B * a.nbands * a.ntiles);
    // the backward's single-direction passes: plain weighted sums of exp
    const bool plain = a.P == nullptr && a.gP == nullptr && !a.times_c &&
                       a.elem_out == nullptr && a.epi == EPI_RAW && a.skip == nullptr &&
                       !a.precise;
    if (vec4 && plain && a.row_q > 0 && a.col_q == 0 && a.v == nullptr && a.alpha == nullptr &&
        a.wr == nullptr) {
        const bool four = a.M <= 1024;
        const int rw = four ? 4 : 2;
        const int64_t groups = a.B * ((a.N + rw - 1) / rw);
        const int64_t want = (groups + kRowThreads / 32 - 1) / (kRowThreads / 32);
        const unsigned g = (unsigned)std::max<int64_t>(1, std::min<int64_t>(want, 148 * 3));
        if (four) k_band_rows<4, 1><<<g, kRowThreads, 0, s>>>(a);
        else k_band_rows<2, 2><<<g, kRowThreads, 0, s>>>(a);
    } else if (vec4 && plain && a.col_q > 0 && a.row_q == 0 && a.u == nullptr &&
               a.beta == nullptr && a.wc == nullptr) {
        k_band_cols<4><<<grid, kColThreads, 0, s>>>(a);
    } else if (a.precise) {
        if (vec4) k_band<4, true><<<grid, kColThreads, 0, s>>>(a);
        else k_band<1, true><<<grid, kColThreads, 0, s>>>(a);
    } else if (vec4) {
        k_band<4><<<grid, kColThreads, 0, s>>>(a);
    } else {
        k_band<1><<<grid, kColThreads, 0, s>>>(a);
    }
    SK_LAUNCHED("k_band launch");
    return SK_OK;
}

}  // namespace sk

using namespace sk;

extern "C" {

int sk_transport_plan(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                      int64_t sCn, int64_t sCm, const float* f, const float* g,
                      double epsilon, const uint8_t* mask_a, const uint8_t* mask_b,
                      float* P, void* stream) {
    clear_error();
    if (int e = check_problem(C, B, N, M, epsilon)) return e;
    if (!f || !g || !P) return fail(SK_ERR_ARG, "f, g and P must be non-NULL");
    PlanArgs a{C, sCb, sCn, sCm, B, N, M, f, g, mask_a, mask_b, (float)(1.0 / epsilon), P, 0};
    const bool v4 = vec4_ok(C, B, M, sCb, sCn, sCm) && dense_ok(P, M) &&
                    ((uintptr_t)g % 16 == 0) &&
                    (mask_b == nullptr || (uintptr_t)mask_b % 4 == 0);
    const int vec = v4 ? 4 : 1;
    a.nchunks = (M + (int64_t)kPlanThreads * vec - 1) / ((int64_t)kPlanThreads * vec);
    const int64_t grid = B * N * a.nchunks;
    if (grid > 0x7fffffffLL) return fail(SK_ERR_ARG, "problem too large for one launch");
    cudaStream_t s = (cudaStream_t)stream;
    if (v4) k_plan<4><<<(unsigned)grid, kPlanThreads, 0, s>>>(a);
    else k_plan<1><<<(unsigned)grid, kPlanThreads, 0, s>>>(a);
    SK_LAUNCHED("k_plan launch");
    return SK_OK;
}

size_t sk_cost_workspace_bytes(int64_t B, int64_t N, int64_t M) {
    if (B <= 0 || N <= 0 || M <= 0) return 0;
    return align_up(sizeof(float) * B * N) +
           std::max(band_workspace_bytes(B, N, M), plan_sums_bytes(B, N, M, false));
}

int sk_cost(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb, int64_t sCn,
            int64_t sCm, const float* f, const float* g, double epsilon, float* out,
            void* workspace, size_t workspace_bytes, void* stream) {
    clear_error();
    if (int e = check_problem(C, B, N, M, epsilon)) return e;
    if (!f || !g || !out) return fail(SK_ERR_ARG, "f, g and out must be non-NULL");
    if (!workspace || workspace_bytes < sk_cost_workspace_bytes(B, N, M))
        return fail(SK_ERR_WORKSPACE, "workspace smaller than sk_cost_workspace_bytes");
    cudaStream_t s = (cudaStream_t)stream;
    float* rows = (float*)workspace;
    void* bws = (char*)workspace + align_up(sizeof(float) * B * N);
    // row sums of P * C (masks ignored, as the reference's cost): the
    // persistent plan pass, or the band pass for layouts it does not take
    const int e0 = plan_sums(C, B, N, M, sCb, sCn, sCm, f, g, epsilon, nullptr, nullptr,
                             nullptr, nullptr, false, rows, nullptr, nullptr, nullptr, bws, s,
                             true);
    if (e0 != kPlanSumsUnsuited) {
        if (e0 != SK_OK) return e0;
    } else {
        BandArgs a = band_base(C, B, N, M, sCb, sCn, sCm, epsilon);
        a.u = f;
        a.v = g;
        a.times_c = 1;
        a.row_q = 1;
        a.row_out1 = rows;
        if (int e = launch_band(a, vec4_ok(C, B, M, sCb, sCn, sCm), bws, s)) return e;
    }
    k_batch_sum<<<(unsigned)B, 256, 0, s>>>(rows, N, out);
    SK_LAUNCHED("k_batch_sum launch");
    return SK_OK;
}

size_t sk_marginal_error_workspace_bytes(int64_t B, int64_t N, int64_t M) {
    if (B <= 0 || N <= 0 || M <= 0) return 0;
    return align_up(sizeof(float) * B * N) + align_up(sizeof(float) * B * M) +
           std::max(band_workspace_bytes(B, N, M), plan_sums_bytes(B, N, M, false));
}

int sk_marginal_error(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                      int64_t sCn, int64_t sCm, const float* f, const float* g, const float* a,
                      const float* b, double epsilon, const uint8_t* mask_a,
                      const uint8_t* mask_b, float* out, void* workspace,
                      size_t workspace_bytes, void* stream) {
    clear_error();
    if (int e = check_problem(C, B, N, M, epsilon)) return e;
    if (!f || !g || !a || !b || !out)
        return fail(SK_ERR_ARG, "f, g, a, b and out must be non-NULL");
    if (!workspace || workspace_bytes < sk_marginal_error_workspace_bytes(B, N, M))
        return fail(SK_ERR_WORKSPACE, "workspace smaller than sk_marginal_error_workspace_bytes");
    cudaStream_t s = (cudaStream_t)stream;
    float* rows = (float*)workspace;
    float* cols = (float*)((char*)workspace + align_up(sizeof(float) * B * N));
    void* bws = (char*)cols + align_up(sizeof(float) * B * M);
    // row and column sums of the masked plan in one pass over C: the
    // persistent plan pass, or the band pass for layouts it does not take
    const int e0 = plan_sums(C, B, N, M, sCb, sCn, sCm, f, g, epsilon, mask_a, mask_b, nullptr,
                             nullptr, false, rows, nullptr, cols, nullptr, bws, s);
    if (e0 != kPlanSumsUnsuited) {
        if (e0 != SK_OK) return e0;
    } else {
        BandArgs ba = band_base(C, B, N, M, sCb, sCn, sCm, epsilon);
        ba.u = f;
        ba.v = g;
        ba.mask_a = mask_a;
        ba.mask_b = mask_b;
        ba.row_q = 1;
        ba.col_q = 1;
        ba.row_out1 = rows;
        ba.col_out1 = cols;
        if (int e = launch_band(ba, vec4_ok(C, B, M, sCb, sCn, sCm), bws, s)) return e;
    }
    SK_CUDA(cudaMemsetAsync(out, 0, sizeof(float), s));
    const int64_t n = B * (N + M);
    const unsigned grid = (unsigned)std::min<int64_t>((n + 255) / 256, 148 * 4);
    k_marginal_err<<<grid, 256, 0, s>>>(rows, cols, a, b, mask_a, mask_b, B * N, B * M, out);
    SK_LAUNCHED("k_marginal_err launch");
    return SK_OK;
}

// the JVP's finished sums (2 row and 2 column vectors) ahead of the pass's own
static size_t jvp_sums_bytes(int64_t B, int64_t N, int64_t M) {
    return 2 * align_up(sizeof(float) * B * N) + 2 * align_up(sizeof(float) * B * M);
}

size_t sk_jvp_workspace_bytes(int64_t B, int64_t N, int64_t M) {
    if (B <= 0 || N <= 0 || M <= 0) return 0;
    return std::max(band_workspace_bytes(B, N, M),
                    jvp_sums_bytes(B, N, M) + plan_sums_bytes(B, N, M, true));
}

int sk_jvp(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb, int64_t sCn,
           int64_t sCm, const float* f, const float* g, double epsilon, const float* v_f,
           const float* v_g, double rho_a, double rho_b, float* out_f, float* out_g,
           void* workspace, size_t workspace_bytes, void* stream) {
    clear_error();
    if (int e = check_problem(C, B, N, M, epsilon)) return e;
    if (!f || !g || !v_f || !v_g || !out_f || !out_g)
        return fail(SK_ERR_ARG, "f, g, v_f, v_g, out_f and out_g must be non-NULL");
    if (!workspace || workspace_bytes < sk_jvp_workspace_bytes(B, N, M))
        return fail(SK_ERR_WORKSPACE, "workspace smaller than sk_jvp_workspace_bytes");
    {
        // the persistent plan pass: P v_g, P 1, P^T v_f, P^T 1, then the mix
        cudaStream_t s = (cudaStream_t)stream;
        char* w = (char*)workspace;
        float* r0 = (float*)w;
        float* r1 = (float*)(w + align_up(sizeof(float) * B * N));
        float* c0 = (float*)(w + 2 * align_up(sizeof(float) * B * N));
        float* c1 = (float*)((char*)c0 + align_up(sizeof(float) * B * M));
        const int e0 = plan_sums(C, B, N, M, sCb, sCn, sCm, f, g, epsilon, nullptr, nullptr,
                                 v_g, v_f, true, r0, r1, c0, c1,
                                 w + jvp_sums_bytes(B, N, M), s);
        if (e0 != kPlanSumsUnsuited) {
            if (e0 != SK_OK) return e0;
            const unsigned gn = (unsigned)std::min<int64_t>((B * N + 255) / 256, 148 * 8);
            const unsigned gm = (unsigned)std::min<int64_t>((B * M + 255) / 256, 148 * 8);
            k_jvp_tail<<<gn, 256, 0, s>>>(r0, r1, v_f, B * N, (float)rho_a,
                                          (float)(1.0 - rho_a), out_f);
            k_jvp_tail<<<gm, 256, 0, s>>>(c0, c1, v_g, B * M, (float)rho_b,
                                          (float)(1.0 - rho_b), out_g);
            SK_LAUNCHED("k_jvp_tail launch");
            return SK_OK;
        }
    }
    BandArgs a = band_base(C, B, N, M, sCb, sCn, sCm, epsilon);
    a.u = f;
    a.v = g;
    a.wr = v_f;
    a.wc = v_g;
    a.row_q = 2;
    a.col_q = 2;
    a.row_out0 = out_f;
    a.col_out0 = out_g;
    a.epi = EPI_JVP;
    a.rho_a = (float)rho_a;
    a.omr_a = (float)(1.0 - rho_a);
    a.rho_b = (float)rho_b;
    a.omr_b = (float)(1.0 - rho_b);
    return launch_band(a, vec4_ok(C, B, M, sCb, sCn, sCm), workspace, (cudaStream_t)stream);
}

int sk_jvp_plan(const float* P, int64_t B, int64_t N, int64_t M, const float* v_f,
                const float* v_g, double rho_a, double rho_b, float* out_f, float* out_g,
                void* workspace, size_t workspace_bytes, void* stream) {
    clear_error();
    if (int e = check_problem(P, B, N, M, 1.0)) return e;
    if (!v_f || !v_g || !out_f || !out_g)
        return fail(SK_ERR_ARG, "v_f, v_g, out_f and out_g must be non-NULL");
    if (!workspace || workspace_bytes < sk_jvp_workspace_bytes(B, N, M))
        return fail(SK_ERR_WORKSPACE, "workspace smaller than sk_jvp_workspace_bytes");
    BandArgs a = band_base(P, B, N, M, N * M, M, 1, 1.0);
    a.P = P;
    a.wr = v_f;
    a.wc = v_g;
    a.row_q = 2;
    a.col_q = 2;
    a.row_out0 = out_f;
    a.col_out0 = out_g;
    a.epi = EPI_JVP;
    a.rho_a = (float)rho_a;
    a.omr_a = (float)(1.0 - rho_a);
    a.rho_b = (float)rho_b;
    a.omr_b = (float)(1.0 - rho_b);
    return launch_band(a, dense_ok(P, M), workspace, (cudaStream_t)stream);
}

int sk_plan_backward(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                     int64_t sCn, int64_t sCm, const float* f, const float* g,
                     double epsilon, const uint8_t* mask_a, const uint8_t* mask_b,
                     const float* grad_P, float* dC, float* df, float* dg,
                     void* workspace, size_t workspace_bytes, void* stream) {
    clear_error();
    if (int e = check_problem(C, B, N, M, epsilon)) return e;
    if (!f || !g || !grad_P) return fail(SK_ERR_ARG, "f, g and grad_P must be non-NULL");
    if (!workspace || workspace_bytes < sk_jvp_workspace_bytes(B, N, M))
        return fail(SK_ERR_WORKSPACE, "workspace smaller than sk_jvp_workspace_bytes");
    BandArgs a = band_base(C, B, N, M, sCb, sCn, sCm, epsilon);
    a.u = f;
    a.v = g;
    a.gP = grad_P;
    a.mask_a = mask_a;
    a.mask_b = mask_b;
    a.scale = (float)(1.0 / epsilon);
    a.elem_out = dC;
    a.elem_scale = -1.f;
    a.row_q = df ? 1 : 0;
    a.col_q = dg ? 1 : 0;
    a.row_out1 = df;
    a.col_out1 = dg;
    const bool v4 = vec4_ok(C, B, M, sCb, sCn, sCm) && dense_ok(grad_P, M) && dense_ok(dC, M);
    return launch_band(a, v4, workspace, (cudaStream_t)stream);
}

}  // extern "C"
