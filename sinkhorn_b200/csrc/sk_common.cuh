// sk_common.cuh -- device helpers shared by the Sinkhorn kernels (sm_100a).
//
// Numerics: a term of the reference, x = (v - c)/eps, is formed in natural
// units as (v - c) * (1/eps), exactly as rounded as the reference's own; the
// running max m stays in natural units and only the small difference x - m is
// scaled by log2(e) before the MUFU ex2, so the shift adds no rounding at large
// |x|. An LSE is m + log(s) with s = sum 2^((x - m) log2 e).
#pragma once

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace sk {

constexpr float kLog2e = 1.44269504088896340736f;
// The reference clamps marginals at 1e-38 before the log (an fp32 subnormal);
// these kernels are built without flush-to-zero so the clamp survives.
constexpr float kTiny = 1e-38f;

// Row-sweep / column-sweep launch shapes.
constexpr int kRowThreads = 256;     // threads per row-sweep CTA
constexpr int kColCT = 32;           // column threads per column-sweep CTA (one warp wide)
constexpr int kColRL = 8;            // row lanes per column-sweep CTA
constexpr int kColThreads = kColCT * kColRL;
constexpr int kColChunk = 8;         // rows a column thread keeps in registers
constexpr int kFinThreads = 256;

// Device status word shared by the kernels of one solve. Lives at the start
// of the workspace; written by the init kernel, read by every sweep.
struct Status {
    int iter;           // index of the iteration being run (0-based)
    int done;           // 1 once converged or max_iters reached: sweeps return
    int n_iters;        // iterations run when done
    int converged;      // 1 if the threshold test passed
    unsigned res_bits;  // max |delta| of the current check iteration (float bits)
    unsigned ticket;    // finalize CTAs done in this iteration
    int max_iters;
    int check_every;    // 0: never check
    float threshold;
    int decide;         // 1: take the convergence decision on the device
    int err;            // nonzero: a kernel detected an inconsistency
    unsigned bar_count;    // on-chip solver: grid-barrier arrivals
    unsigned bar_gen;      // on-chip solver: grid-barrier generation
    unsigned res_slot[3];  // on-chip solver: batch residual per check (float bits)
};
static_assert(sizeof(Status) == 64, "Status is one 64-byte record");

// The status region of a workspace is 256 bytes: the Status record at 0 and
// the persistent solve's grid-barrier arrival counter alone on the cache line
// at byte 128 (so waiters polling it do not contend with the record).
__host__ __device__ inline unsigned* status_bar(void* status) {
    return reinterpret_cast<unsigned*>(reinterpret_cast<char*>(status) + 128);
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Programmatic dependent launch. Every iteration kernel starts with
// pdl_wait(): it returns once the previous kernel on the stream has completed
// and its memory is visible (at once when the launch was not programmatic),
// so no kernel touches its predecessor's results early. pdl_trigger() then
// lets the next kernel's CTAs be scheduled while this one still runs; they
// wait in their own pdl_wait(). Together they hide the launch gap between
// consecutive iteration kernels.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// exp(d) for d <= 0 (a shifted LSE term): one MUFU op
__device__ __forceinline__ float expd(float d) { return ex2(d * kLog2e); }

constexpr float kLn2 = 0.69314718055994530942f;

// exp(d / eps) to a few ulp, given K = log2(e) / eps as the pair khi + klo
// (khi the float nearest K, klo the float nearest K - khi). The product d * K
// is carried as y + ylo: the FMA gives the exact rounding error of d * khi
// (Dekker's product), d * klo adds the error of khi. 2^y comes from
// ex2.approx, and 2^ylo = 1 + ylo ln2 + O(ylo^2) is applied as a first-order
// correction (|ylo| is at most about ulp(y)). The correction is clamped to
// [-1/4, 1/4]: it is far smaller for every finite argument, and for an
// infinite one (NaN correction) the clamp keeps exp(-inf) = 0 and
// exp(inf) = inf, while a NaN argument stays NaN through 2^y. Unlike
// expd, the argument's own rounding (d * 1/eps * log2e, up to |y| * 2^-23
// relative) does not reach the result.
__device__ __forceinline__ float exp_scaled(float d, float khi, float klo) {
    const float y = d * khi;
    float ylo = fmaf(d, khi, -y);
    ylo = fmaf(d, klo, ylo);
    const float e = ex2(y);
    const float corr = fmaxf(fminf(ylo * kLn2, 0.25f), -0.25f);
    return fmaf(e, corr, e);
}

// Merge the running pair (m, s) -- max (natural units) and sum of exp(x-m) --
// with (m2, s2). Two empty pairs (m = -inf) stay empty.
__device__ __forceinline__ void lse_merge(float& m, float& s, float m2, float s2) {
    float mn = fmaxf(m, m2);
    if (mn == -INFINITY) return;
    s = s * expd(m - mn) + s2 * expd(m2 - mn);
    m = mn;
}

// Fold K new terms into (m, s) with one max pass and K + 1 exponentials.
template <int K>
__device__ __forceinline__ void lse_fold(float& m, float& s, const float (&x)[K]) {
    float cm = x[0];
#pragma unroll
    for (int q = 1; q < K; ++q) cm = fmaxf(cm, x[q]);
    if (cm == -INFINITY) return;  // every term empty (masked / padding)
    float mn = fmaxf(m, cm);
    float acc = 0.f;
#pragma unroll
    for (int q = 0; q < K; ++q) acc += expd(x[q] - mn);
    s = s * expd(m - mn) + acc;
    m = mn;
}

// lse_fold on the packed fp32x2 pipe, terms in pairs: the same per-term
// rounding (x - mn, * log2 e, ex2), two partial sums added at the end.
template <int K2>
__device__ __forceinline__ void lse_fold_pairs(float& m, float& s, const float2 (&x)[K2]) {
    float cm = fmaxf(x[0].x, x[0].y);
#pragma unroll
    for (int q = 1; q < K2; ++q) cm = fmaxf(cm, fmaxf(x[q].x, x[q].y));
    if (cm == -INFINITY) return;  // every term empty (masked / padding)
    const float mn = fmaxf(m, cm);
    const float2 nmn = make_float2(-mn, -mn), l2e = make_float2(kLog2e, kLog2e);
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int q = 0; q < K2; ++q) {
        const float2 d = __fmul2_rn(__fadd2_rn(x[q], nmn), l2e);
        acc = __fadd2_rn(acc, make_float2(ex2(d.x), ex2(d.y)));
    }
    s = s * expd(m - mn) + (acc.x + acc.y);
    m = mn;
}

// Two independent lse_folds (two columns) side by side on the packed pipe;
// each column's terms are folded in the same order and rounded the same way
// as lse_fold does it.
template <int K>
__device__ __forceinline__ void lse_fold_x2(float& ma, float& sa, float& mb, float& sb,
                                            const float (&xa)[K], const float (&xb)[K]) {
    float ca = xa[0], cb = xb[0];
#pragma unroll
    for (int q = 1; q < K; ++q) {
        ca = fmaxf(ca, xa[q]);
        cb = fmaxf(cb, xb[q]);
    }
    const bool ea = ca == -INFINITY, eb = cb == -INFINITY;  // every term empty
    if (ea && eb) return;
    const float2 mn = make_float2(fmaxf(ma, ca), fmaxf(mb, cb));
    const float2 nmn = make_float2(-mn.x, -mn.y), l2e = make_float2(kLog2e, kLog2e);
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int q = 0; q < K; ++q) {
        const float2 d = __fmul2_rn(__fadd2_rn(make_float2(xa[q], xb[q]), nmn), l2e);
        acc = __fadd2_rn(acc, make_float2(ex2(d.x), ex2(d.y)));
    }
    const float2 dm = __fmul2_rn(__fadd2_rn(make_float2(ma, mb), nmn), l2e);
    const float2 ns = __ffma2_rn(make_float2(sa, sb), make_float2(ex2(dm.x), ex2(dm.y)), acc);
    if (!ea) {
        ma = mn.x;
        sa = ns.x;
    }
    if (!eb) {
        mb = mn.y;
        sb = ns.y;
    }
}

// (g - c) * k for a pair, rounded as the scalar form (g - c as fma(c, -1, g)).
__device__ __forceinline__ float2 scaled_diff2(float2 g, float2 c, float k) {
    return __fmul2_rn(__ffma2_rn(c, make_float2(-1.f, -1.f), g), make_float2(k, k));
}

__device__ __forceinline__ void warp_lse_reduce(float& m, float& s, int width = 32) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        if (o < width) {
            float m2 = __shfl_xor_sync(0xffffffffu, m, o);
            float s2 = __shfl_xor_sync(0xffffffffu, s, o);
            lse_merge(m, s, m2, s2);
        }
    }
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Residual max of non-negative floats (NaN compares above +inf as bits, so a
// NaN residual never passes the threshold test).
__device__ __forceinline__ void atomic_max_nonneg(unsigned* p, float v) {
    atomicMax(p, __float_as_uint(v));
}

// Streaming 128-bit load of C: not kept in L1 (each element is used once per
// sweep), default L2 policy so small problems stay L2-resident across sweeps.
__device__ __forceinline__ float4 ld_stream4(const float* p) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ float ld_stream1(const float* p) {
    float v;
    asm volatile("ld.global.nc.L1::no_allocate.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}

// C element types: fp32, or bf16 carried as its 16-bit pattern (uint16_t).
// A bf16 value widens to fp32 exactly: its bits are the fp32's top 16.
__device__ __forceinline__ float4 bf16x4_to_float4(uint32_t lo, uint32_t hi) {
    return make_float4(__uint_as_float(lo << 16), __uint_as_float(lo & 0xffff0000u),
                       __uint_as_float(hi << 16), __uint_as_float(hi & 0xffff0000u));
}

// Four consecutive elements of C as fp32, streaming (not kept in L1).
template <typename T>
__device__ __forceinline__ float4 ld_c4(const T* p);
template <>
__device__ __forceinline__ float4 ld_c4<float>(const float* p) {
    return ld_stream4(p);
}
template <>
__device__ __forceinline__ float4 ld_c4<uint16_t>(const uint16_t* p) {
    uint32_t lo, hi;
    asm volatile("ld.global.nc.L1::no_allocate.v2.b32 {%0,%1}, [%2];"
                 : "=r"(lo), "=r"(hi)
                 : "l"(p));
    return bf16x4_to_float4(lo, hi);
}

// One element of C as fp32, streaming.
template <typename T>
__device__ __forceinline__ float ld_c1(const T* p);
template <>
__device__ __forceinline__ float ld_c1<float>(const float* p) {
    return ld_stream1(p);
}
template <>
__device__ __forceinline__ float ld_c1<uint16_t>(const uint16_t* p) {
    unsigned short v;
    asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return __uint_as_float((uint32_t)v << 16);
}

// Four consecutive elements of a shared-memory copy of C as fp32.
template <typename T>
__device__ __forceinline__ float4 lds_c4(const T* p);
template <>
__device__ __forceinline__ float4 lds_c4<float>(const float* p) {
    return *reinterpret_cast<const float4*>(p);
}
template <>
__device__ __forceinline__ float4 lds_c4<uint16_t>(const uint16_t* p) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    return bf16x4_to_float4(v.x, v.y);
}

// Vector loaded through L1 (potentials reused by every row / column).
__device__ __forceinline__ float4 ld_vec4(const float* p) {
    return __ldg(reinterpret_cast<const float4*>(p));
}

__device__ __forceinline__ int read_volatile(const int* p) {
    return *reinterpret_cast<const volatile int*>(p);
}

__device__ __forceinline__ float lse_of(float m, float s) {
    return (m == -INFINITY) ? -INFINITY : m + logf(s);
}

// Softmin epilogue shared by every update: softmin = -eps*(m + log s), 0 for
// an empty set (lse_kernel.py:130,206) and, when `guard` is set, 0 for any
// infinite value (forward.py:41,76).
__device__ __forceinline__ float softmin_from_pair(float m, float s, float eps,
                                                  bool guard) {
    if (m == -INFINITY) return 0.f;
    float sm = -eps * (m + logf(s));
    if (guard && isinf(sm)) sm = 0.f;
    return sm;
}

}  // namespace sk
