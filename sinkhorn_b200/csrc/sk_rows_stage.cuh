// sk_rows_stage.cuh -- the role layout shared by the whole-row single-read
// kernels (k_rows_fused, the forward iteration for 512 <= M <= 2048, and
// k_bwd_rows, the backward's reverse step on the same shapes): a producer
// warp streams row groups into a shared-memory ring with bulk copies, 16
// consumer warps reduce each stage's rows and fold the previous stage into
// per-column sums, and a finisher warp turns the rows' sums into per-row
// values. The roles meet on mbarriers only, and every wait is bounded.
#pragma once

#include "sk_common.cuh"
#include "sk_internal.h"
#include "sk_tma.cuh"

namespace sk {

constexpr int kRfWarps = 16;                     // consumer warps
constexpr int kRfConsumers = 32 * kRfWarps;      // 512 consumer threads
constexpr int kRfProducer = kRfWarps;            // warp 16
constexpr int kRfFinisher = kRfWarps + 1;        // warp 17
constexpr int kRfThreads = kRfConsumers + 64;    // + producer and finisher warps
constexpr int kRfSetRows = 4;                    // rows of the ring's unit set (see rf_stages)
constexpr int kRfMaxRows = 32;                   // rows per stage (8 per thread, TPC = 4)
constexpr int kRfStages = 6;
constexpr int kRfMinM = 512, kRfMaxM = 2048;

// threads per column group: 1 up to M = 2048, 2 up to 1024, 4 up to 512
inline int rf_tpc(int64_t M) { return M <= 512 ? 4 : (M <= 1024 ? 2 : 1); }

// the ring's bytes: kRfStages x kRfSetRows x TPC rows of M floats (laid out
// as rf_stages() stages of rf_set_rows() x TPC rows)
inline size_t rf_ring_bytes(int64_t M) {
    return sizeof(float) * (size_t)kRfStages * kRfSetRows * rf_tpc(M) * M;
}

__device__ __forceinline__ void rf_consumers_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kRfConsumers) : "memory");
}

// Bounded wait that gives up early once another role has aborted.
__device__ __forceinline__ bool rf_wait(uint64_t* bar, uint32_t parity, volatile int* ab) {
    for (uint32_t i = 0; i < kWaitPolls; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*ab) return false;
    }
    return false;
}

__device__ __forceinline__ void rf_abort(volatile int* ab, Status* st) {
    *ab = 1;
    atomicMax(&st->err, 2);
}

// One butterfly stage of the transposed reduction for plain sums: lanes whose
// `bit` is set keep the upper half of their n sums and send the lower half
// across `off`.
template <int n>
__device__ __forceinline__ void rf_halve_sum(const float (&s)[2 * n], float (&os)[n], bool hi,
                                             int off) {
#pragma unroll
    for (int i = 0; i < n; ++i) {
        const float ks = hi ? s[i + n] : s[i], ss = hi ? s[i] : s[i + n];
        os[i] = ks + __shfl_xor_sync(0xffffffffu, ss, off);
    }
}

// A warp's 4 per-row sums (one set per lane) added over the warp: lanes
// 8 r .. 8 r + 7 end with row r's total.
__device__ __forceinline__ float rf_warp_rows4(const float (&ps)[kRfSetRows], int lane) {
    float as[2], bs[1];
    rf_halve_sum<2>(ps, as, (lane & 16) != 0, 16);
    rf_halve_sum<1>(as, bs, (lane & 8) != 0, 8);
    float s2 = bs[0];
    s2 += __shfl_xor_sync(0xffffffffu, s2, 4);
    s2 += __shfl_xor_sync(0xffffffffu, s2, 2);
    s2 += __shfl_xor_sync(0xffffffffu, s2, 1);
    return s2;
}

// The same for 8 per-row sums: lanes 4 r .. 4 r + 3 end with row r's total.
__device__ __forceinline__ float rf_warp_rows8(const float (&ps)[8], int lane) {
    float a4[4], a2[2], a1[1];
    rf_halve_sum<4>(ps, a4, (lane & 16) != 0, 16);
    rf_halve_sum<2>(a4, a2, (lane & 8) != 0, 8);
    rf_halve_sum<1>(a2, a1, (lane & 4) != 0, 4);
    float s2 = a1[0];
    s2 += __shfl_xor_sync(0xffffffffu, s2, 2);
    s2 += __shfl_xor_sync(0xffffffffu, s2, 1);
    return s2;
}

// Rows per thread and stage of the whole-row kernels: 8 (R = 8 TPC rows per
// stage in 3 stages, the ring bytes of 6 stages of 4-row sets), so a thread's
// per-stage work (waits, hand-offs, the warp butterfly) is spread over 32
// elements; measured against 4 rows per thread: B=16 N=M=2048 78.7 -> 63.8
// us per iteration, B=64 N=2048 M=512 97.4 -> 88.0 us.
template <int TPC>
constexpr int rf_set_rows() {
    return 8;
}
template <int TPC>
constexpr int rf_stages() {
    return kRfStages * kRfSetRows / rf_set_rows<TPC>();
}

}  // namespace sk
