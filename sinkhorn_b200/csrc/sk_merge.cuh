// sk_merge.cuh -- merging partial column LSEs in one fixed order.
//
// The g-update of a single-read iteration merges, for every column, P partial
// LSEs (natural log; -inf: no term): one per row chunk on one GPU, one per
// rank in a row-sharded solve. Every kernel that does this merge -- the
// k_col_finish launch and the merge phase of the persistent solve -- uses the
// functions below, so their results are bit-identical whatever kernel ran:
//   * the partials are split into kMergeSubsets interleaved subsets
//     (p = s, s + 4, s + 8, ...); one thread per (column, subset) loads its
//     subset's values (up to kMergeHeld of them at once, all loads in
//     flight) and folds them kMergeBatch at a time in increasing p;
//   * the subset pairs are then merged in subset order 0, 1, 2, 3.
// The loads are the latency of the merge (the partials sit in L2), so the
// point of the layout is that a thread waits for one round trip, not one per
// partial.
#pragma once

#include <math.h>
#include <stdint.h>

#include "sk_common.cuh"

namespace sk {

constexpr int kMergeSubsets = 4;
constexpr int kMergeBatch = 8;
constexpr int kMergeHeld = 32;  // values per thread loaded before folding

// Partial value p of a column: through L2 only (CG = true, for data written
// earlier in the same launch) or the read-only path.
template <bool CG>
__device__ __forceinline__ float merge_load(const float* p) {
    if constexpr (CG) return __ldcg(p);
    else return __ldg(p);
}

// (max, sum) pair of subset s of the P partials src[p * stride] (natural log
// units; sum of exp(v - max)). live = false gives the empty pair.
template <bool CG>
__device__ __forceinline__ float2 merge_subset(const float* src, int64_t stride, int P, int s,
                                               bool live) {
    float mm = -INFINITY, ss = 0.f;
    if (!live) return make_float2(mm, ss);
    for (int p0 = s; p0 < P; p0 += kMergeSubsets * kMergeHeld) {
        float v[kMergeHeld];
#pragma unroll
        for (int k = 0; k < kMergeHeld; ++k) {
            const int p = p0 + kMergeSubsets * k;
            v[k] = p < P ? merge_load<CG>(src + (int64_t)p * stride) : -INFINITY;
        }
#pragma unroll
        for (int k = 0; k < kMergeHeld; k += kMergeBatch) {
            float w[kMergeBatch];
#pragma unroll
            for (int q = 0; q < kMergeBatch; ++q) w[q] = v[k + q];
            lse_fold<kMergeBatch>(mm, ss, w);
        }
    }
    return make_float2(mm, ss);
}

// Merge subset pairs 1..3 into subset 0's pair, in subset order.
__device__ __forceinline__ void merge_subsets(float& mm, float& ss,
                                              const float2 (&sub)[kMergeSubsets]) {
    mm = sub[0].x;
    ss = sub[0].y;
#pragma unroll
    for (int s = 1; s < kMergeSubsets; ++s) lse_merge(mm, ss, sub[s].x, sub[s].y);
}

}  // namespace sk
