// sk_api.cpp -- error reporting, planning and workspace layout of the C ABI.
#include <stdio.h>

#include <algorithm>
#include <cmath>
#include <string>

#include "sk_internal.h"

namespace sk {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }
void clear_error() { g_last_error.clear(); }

int fail(int code, const std::string& msg) {
    set_error(msg);
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    std::string m = std::string(what) + ": " + cudaGetErrorName(e) + " (" +
                    cudaGetErrorString(e) + ")";
    set_error(m);
    return SK_ERR_CUDA;
}

constexpr int64_t kSMs = 148;
constexpr int64_t kColTargetCtas = kSMs * 8 * 4;
constexpr int64_t kBandQuantum = 64;  // kColRL * kColChunk

int64_t col_bands(int64_t B, int64_t N, int64_t M, int64_t* band_rows) {
    const int64_t tiles = (M + 127) / 128;
    const int64_t items = std::max<int64_t>(1, tiles * B);
    int64_t nb = (kColTargetCtas + items - 1) / items;
    const int64_t max_nb = std::max<int64_t>(1, (N + kBandQuantum - 1) / kBandQuantum);
    nb = std::min(std::max<int64_t>(nb, 1), max_nb);
    int64_t br = (N + nb - 1) / nb;
    br = std::max<int64_t>(kBandQuantum, (br + kBandQuantum - 1) / kBandQuantum * kBandQuantum);
    nb = std::max<int64_t>(1, (N + br - 1) / br);
    if (band_rows) *band_rows = br;
    return nb;
}

int64_t max_col_tiles(int64_t M) { return (M + 31) / 32; }

SweepPlan make_plan(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                    int64_t sCn, int64_t sCm) {
    SweepPlan p;
    const bool aligned = ((uintptr_t)C % 16 == 0) && sCm == 1 && M % 4 == 0 &&
                         sCn % 4 == 0 && (B == 1 || sCb % 4 == 0);
    p.vec = aligned ? 4 : 1;
    p.nbands = col_bands(B, N, M, &p.band_rows);
    const int64_t tj = 32 * p.vec;
    p.ntiles = (M + tj - 1) / tj;
    // row-sweep threads per row: ~16 vector loads per thread
    const int64_t nv = (M + p.vec - 1) / p.vec;
    int tpr = 32;
    while (tpr < 256 && (int64_t)tpr * 2 <= nv / 16) tpr *= 2;
    p.tpr = tpr;
    p.fused = 0;
    p.fused_ok = 0;
    p.col_tma = p.vec == 4 ? 1 : 0;
    if (p.col_tma) {
        // the tensor-fed sweep runs 2 CTAs per SM; long bands keep its ring
        // streaming (about 4 waves of 296 CTAs), never more bands than the
        // workspace was sized for
        const int64_t items = std::max<int64_t>(1, B * p.ntiles);
        int64_t nb = std::max<int64_t>(1, (kSMs * 3 * 4 + items - 1) / items);
        nb = std::min(nb, p.nbands);
        int64_t br = (N + nb - 1) / nb;
        br = (br + kBandQuantum - 1) / kBandQuantum * kBandQuantum;
        p.band_rows = br;
        p.nbands = (N + br - 1) / br;
    }
    p.chunks = 0;
    p.rows_per_chunk = 0;
    p.bf16 = 0;
    p.fused_rows = 0;
    p.cluster = 0;
    p.persist = 0;
    p.solve_chunks = 0;
    p.solve_rows = 0;
    if (p.vec == 4) plan_fused(p, B, N, M);
    return p;
}

SweepPlan make_plan_bf16(const float* C, int64_t B, int64_t N, int64_t M, int64_t sCb,
                         int64_t sCn, int64_t sCm) {
    // a 4-element group of bf16 is 8 bytes: the fp32 plan's alignment rules
    // (16-byte base, sCn and sCb multiples of 4 elements) keep groups aligned
    SweepPlan p = make_plan(C, B, N, M, sCb, sCn, sCm);
    if (p.vec != 4) {
        p.vec = 0;
        return p;
    }
    if (p.cluster == 1) plan_fused(p, B, N, M, false);
    p.bf16 = 1;
    p.col_tma = 0;
    p.nbands = col_bands(B, N, M, &p.band_rows);
    // the fused iteration copies half-rows of M/2 bf16 with cp.async.bulk:
    // sizes and every start (b sCb + i sCn + M/2 elements, 2 bytes each) must
    // be 16-byte multiples
    if (M % 16 != 0 || sCn % 8 != 0 || (B > 1 && sCb % 8 != 0) || p.fused_rows ||
        p.cluster != 2) {
        p.fused = 0;  // (k_rows_fused and the 4- / 8-CTA clusters read fp32 C only)
        p.fused_ok = 0;
        p.fused_rows = 0;
    }
    p.persist = 0;  // the persistent solve reads fp32 C only
    return p;
}

SolveWs carve_solve(void* base, int64_t B, int64_t N, int64_t M) {
    SolveWs w{};
    int64_t br = 0;
    const int64_t nb = col_bands(B, N, M, &br);
    char* p = (char*)base;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        char* r = p ? p + off : nullptr;
        off += align_up(bytes);
        return r;
    };
    w.status = take(status_bytes(B * M));  // Status, grid-barrier line, finish counters
    w.log_a = (float*)take(sizeof(float) * B * N);
    w.log_b = (float*)take(sizeof(float) * B * M);
    w.f_eff = (float*)take(sizeof(float) * B * N);
    w.g_eff = (float*)take(sizeof(float) * B * M);
    w.ranges = (int*)take(sizeof(int) * 4 * B);
    w.tickets = (unsigned*)take(sizeof(unsigned) * B * max_col_tiles(M));
    w.partial = (float*)take(sizeof(float) * B * nb * M);
    w.fparts = (float*)take(sizeof(float) * fused_max_chunks(B, N, M) * (B * M + 4));
    w.bytes = off;
    return w;
}

int check_problem(const float* C, int64_t B, int64_t N, int64_t M, double epsilon) {
    if (C == nullptr) return fail(SK_ERR_ARG, "C is NULL");
    if (B <= 0 || N <= 0 || M <= 0)
        return fail(SK_ERR_ARG, "B, N and M must be positive");
    if (!(epsilon > 0.0) || !std::isfinite(epsilon))
        return fail(SK_ERR_ARG, "epsilon must be a positive finite number");
    if (N > (int64_t)1 << 31 || M > (int64_t)1 << 31)
        return fail(SK_ERR_ARG, "N and M must be below 2^31");
    return SK_OK;
}

}  // namespace sk

extern "C" {

int sk_version(void) { return 100; }

const char* sk_last_error(void) { return sk::g_last_error.c_str(); }

}  // extern "C"
