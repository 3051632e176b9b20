// ordered_sum.cuh -- the reference's left-to-right f32 running sum,
// reproduced exactly with warp-parallel integer prefix sums.
//
// The reference softmax (src/ops/softmax.c:15-22) accumulates
//     sum = fl(sum + e_0); sum = fl(sum + e_1); ...   (f32, round to nearest even)
// strictly in index order, with every e_i >= 0.  A tree sum of the same
// terms differs from that by the sequential sum's own rounding error
// (measured up to ~2e-4 relative at 128K terms), so a parallel reduction
// cannot meet a 1e-5 bound against it.  This routine returns the sequential
// sum bit-for-bit while processing 32*K terms per warp step.
//
// Why that is possible.  Let the running sum s lie in the binade
// [2^b, 2^(b+1)) (for s < 2^-126, the subnormal grid: b = -126).  Every f32
// there is a multiple of u = 2^(b-23), so s = S*u for an integer
// S < 2^24.  As long as the result stays in the binade,
//     fl(s + e) = (S + rne(e/u)) * u,
// except when e/u is exactly halfway between integers, where the tie is
// broken by the parity of the result.  e/u is an exact power-of-two scaling,
// so d = rne(e/u) is one multiply and one conversion, and the terms of a
// whole tile add as integers: a warp prefix sum.  The sum is monotone
// (e >= 0), so the binade only grows; an "event" -- the first term whose
// result would reach 2^(b+1), or an exact tie -- is found with a ballot,
// performed as the real f32 addition fl(s_before + e) on the exact s_before
// = run*u, and the scan resumes after it with the new binade.  Binade
// crossings happen about log2(sum/first term) times per row; exact ties are
// rare once s >> e.  For tiny sums (s < 2^-100, where 1/u would overflow)
// the terms are added one by one.  NaN terms make the sum NaN, as in the
// reference.
#pragma once

#include "tb_device.cuh"

namespace tbk {

struct RunSum {
    float s;         // the running sum, bit-identical to the sequential one
    uint32_t S;      // s / u (fast mode)
    float u, inv_u;  // grid spacing of s's binade and its inverse
    int b;           // the binade: s in [2^b, 2^(b+1)) (b = -126 below that)
    bool fast;       // s >= 2^-100: integer-grid mode
    bool nan;        // sum is NaN; nothing more to do

    __device__ __forceinline__ void set(float v) {
        s = v;
        nan = (v != v);
        fast = false;
        b = -127;
        if (nan) return;
        const int ex = (int)(__float_as_uint(v) >> 23) - 127;  // v >= 0
        b = ex < -126 ? -126 : ex;
        if (b >= -100) {
            fast = true;
            u = __uint_as_float((uint32_t)(b - 23 + 127) << 23);
            inv_u = __uint_as_float((uint32_t)(23 - b + 127) << 23);
            S = (uint32_t)__fmul_rn(v, inv_u);
        }
    }
};

// Binade of a positive estimate for the integer-grid mode, or kNoBinade
// when the estimate is below 2^-100, zero, or NaN.
constexpr int kNoBinade = -128;
__device__ __forceinline__ int binade_of(float v) {
    if (!(v >= 7.8886090522101181e-31f)) return kNoBinade;  // 2^-100
    return (int)(__float_as_uint(v) >> 23) - 127;
}

// d = rne(e / u) for the grid 2^(b-23), capped at 2^25 (already an event);
// sets *event for an exact tie (parity-dependent rounding) or a NaN term.
__device__ __forceinline__ uint32_t grid_units(float e, float inv_u, bool* event) {
    const float t = __fmul_rn(e, inv_u);
    if (!(t < 33554432.0f)) {
        if (t != t) *event = true;
        return 1u << 25;
    }
    if (__fsub_rn(t, floorf(t)) == 0.5f) *event = true;
    return __float2uint_rn(t);
}

__device__ __forceinline__ float inv_grid(int b) {
    return __uint_as_float((uint32_t)(23 - b + 127) << 23);
}

// Consume the first `nvalid` terms of a warp tile, in order: lane l holds
// terms l*K .. l*K+K-1 in e[].  All 32 lanes call it with identical `st`
// and leave with identical `st`.
// Terms before `first` are taken as already consumed.
template <int K>
__device__ __forceinline__ void ordered_sum_tile(RunSum& st, const float (&e)[K], int nvalid,
                                                 int first = 0) {
    constexpr uint32_t kLimit = 1u << 24;  // S reaching this leaves the binade
    constexpr uint32_t kCap = 1u << 25;    // any d >= 2^24 is an event anyway
    constexpr uint32_t kSat = 1u << 30;    // saturation of partial sums
    const int lane = threadIdx.x & 31;
    int pos = first;  // terms of this tile already consumed
    while (pos < nvalid && !st.nan) {
        if (!st.fast) {
            // Tiny sum: exact one-by-one additions, in sequence order.
            for (int L = 0; L < 32; ++L) {
#pragma unroll
                for (int kk = 0; kk < K; ++kk) {
                    const float v = __shfl_sync(kFull, e[kk], L);
                    const int p = L * K + kk;
                    if (p >= pos && p < nvalid && !st.fast && !st.nan) {
                        st.set(__fadd_rn(st.s, v));
                        pos = p + 1;
                    }
                }
            }
            if (!st.fast) pos = nvalid;
            continue;
        }
        uint32_t d[K];
        uint32_t tie = 0, lsum = 0;
#pragma unroll
        for (int kk = 0; kk < K; ++kk) {
            const int p = lane * K + kk;
            uint32_t dk = 0;
            if (p >= pos && p < nvalid) {
                const float t = __fmul_rn(e[kk], st.inv_u);
                if (!(t < (float)kCap)) {  // huge, or NaN
                    dk = kCap;
                    if (t != t) tie |= 1u << kk;
                } else {
                    dk = __float2uint_rn(t);
                    if (__fsub_rn(t, floorf(t)) == 0.5f) tie |= 1u << kk;
                }
            }
            d[kk] = dk;
            lsum = min(lsum + dk, kSat);
        }
        uint32_t incl = lsum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t n = __shfl_up_sync(kFull, incl, o);
            if (lane >= o) incl = min(incl + n, kSat);
        }
        uint32_t excl = __shfl_up_sync(kFull, incl, 1);
        if (lane == 0) excl = 0;
        const uint32_t total = __shfl_sync(kFull, incl, 31);
        const bool ev = tie != 0 || (st.S + excl + lsum >= kLimit);
        const unsigned bal = __ballot_sync(kFull, ev);
        if (bal == 0) {
            st.S += total;
            st.s = __fmul_rn((float)st.S, st.u);
            return;
        }
        // First event: lane f, term kstar.  Lanes before f had no event, so
        // S + excl is exact (unsaturated) in lane f.
        const int f = __ffs(bal) - 1;
        float snew = 0.0f;
        int kstar = 0;
        if (lane == f) {
            uint32_t run = st.S + excl;
            bool found = false;
#pragma unroll
            for (int kk = 0; kk < K; ++kk) {
                const int p = lane * K + kk;
                if (!found && p >= pos && p < nvalid) {
                    if (((tie >> kk) & 1u) || run + d[kk] >= kLimit) {
                        found = true;
                        kstar = kk;
                        snew = __fadd_rn(__fmul_rn((float)run, st.u), e[kk]);
                    } else {
                        run += d[kk];
                    }
                }
            }
        }
        snew = __shfl_sync(kFull, snew, f);
        kstar = __shfl_sync(kFull, kstar, f);
        st.set(snew);
        pos = f * K + kstar + 1;
    }
}

}  // namespace tbk
