// gemv.cuh -- per-warp row dot products of the decoder's GEMVs: dense f32
// rows, and 2:4 rows in the packed form of k_sparse24.cu.
//
// A warp takes two output rows at once, so every float4 of x it loads
// (through L1) serves both.  Lanes stride over the row in steps of 128
// float4s (dense) or 128 group pairs (packed), four per lane per row in
// flight, with no bounds checks inside a full step; the last partial step
// goes element by element.  A call may cover a range of steps [s0, s1) so
// several warps can split a row (the range holding the partial step takes
// it).  The result is each lane's partial sum; the caller adds the lanes
// (warp_sum2).
//
// Packed form, per row: P = (in/4)/2 pairs of 4-column groups; vals holds a
// float4 per pair (group 2p's two kept weights, then group 2p+1's) and idx a
// byte per pair (2 bits per slot: the kept column within its group), laid
// out so that one 32-bit load gives a lane its four bytes of a step: the
// byte of pair p = 128 s + 32 u + l is at 128 s + 4 l + u, and a row of idx
// is padded to a multiple of 128 bytes.
#pragma once
#include "tb_device.cuh"

namespace tbk {

constexpr int kGemvStep = 128;  // float4s (dense) or pairs (packed) per warp step

__host__ __device__ inline int64_t packed_idx_stride(int64_t pairs) {
    return (pairs + kGemvStep - 1) / kGemvStep * kGemvStep;
}

// x[4 g + k] for k = the 2-bit field's value.
__device__ __forceinline__ float pick4(const float4& x, uint32_t k) {
    const float lo = (k & 1u) ? x.y : x.x;
    const float hi = (k & 1u) ? x.w : x.z;
    return (k & 2u) ? hi : lo;
}

// The four kept weights of a pair against x columns 8p .. 8p+7.
__device__ __forceinline__ float pair_dot(const float4& v, uint32_t ib, const float4& xa,
                                          const float4& xb, float acc) {
    acc = __fmaf_rn(v.x, pick4(xa, ib), acc);
    acc = __fmaf_rn(v.y, pick4(xa, ib >> 2), acc);
    acc = __fmaf_rn(v.z, pick4(xb, ib >> 4), acc);
    acc = __fmaf_rn(v.w, pick4(xb, ib >> 6), acc);
    return acc;
}

// x through the read-only path from global memory, or from shared memory.
template <bool XS>
__device__ __forceinline__ float4 ldx(const float4* p) {
    if constexpr (XS)
        return *p;
    else
        return __ldg(p);
}

// Partial sums of two packed rows (v0/i0 and v1/i1; pass the same row twice
// for one).  pairs: P.  XS: x4 points to shared memory.
template <bool XS = false>
__device__ __forceinline__ void packed_dot2(const float4* __restrict__ v0,
                                            const uint8_t* __restrict__ i0,
                                            const float4* __restrict__ v1,
                                            const uint8_t* __restrict__ i1, int64_t pairs,
                                            const float4* x4, int lane, float& a0, float& a1,
                                            int64_t s0 = 0, int64_t s1 = -1) {
    // steps [s0, s1) of the row (all of it by default); the partial last
    // step belongs to whoever owns step pairs / 128
    const int64_t full = pairs / kGemvStep;
    if (s1 < 0) s1 = full + 1;
    const int64_t send = s1 < full ? s1 : full;
    const float4* p0 = v0 + s0 * kGemvStep + lane;
    const float4* p1 = v1 + s0 * kGemvStep + lane;
    const uint32_t* q0 = reinterpret_cast<const uint32_t*>(i0 + s0 * kGemvStep) + lane;
    const uint32_t* q1 = reinterpret_cast<const uint32_t*>(i1 + s0 * kGemvStep) + lane;
    const float4* xp = x4 + 2 * (s0 * kGemvStep + lane);
    for (int64_t s = s0; s < send; ++s) {
        float4 w0[4], w1[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            w0[u] = __ldcs(p0 + 32 * u);
            w1[u] = __ldcs(p1 + 32 * u);
        }
        const uint32_t b0 = __ldcs(q0), b1 = __ldcs(q1);
        p0 += kGemvStep;
        p1 += kGemvStep;
        q0 += 32;
        q1 += 32;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const float4 xa = ldx<XS>(xp + 64 * u), xb = ldx<XS>(xp + 64 * u + 1);
            a0 = pair_dot(w0[u], b0 >> (8 * u), xa, xb, a0);
            a1 = pair_dot(w1[u], b1 >> (8 * u), xa, xb, a1);
        }
        xp += 2 * kGemvStep;
    }
    if (s1 <= full) return;
    for (int u = 0; u < 4; ++u) {  // the partial step
        const int64_t p = full * kGemvStep + 32 * u + lane;
        if (p >= pairs) break;
        const float4 xa = ldx<XS>(x4 + 2 * p), xb = ldx<XS>(x4 + 2 * p + 1);
        const int64_t ib = full * kGemvStep + 4 * lane + u;
        a0 = pair_dot(__ldcs(v0 + p), i0[ib], xa, xb, a0);
        a1 = pair_dot(__ldcs(v1 + p), i1[ib], xa, xb, a1);
    }
}

// Partial sums of two dense rows of n4 float4s each.
template <bool XS = false>
__device__ __forceinline__ void dense_dot2(const float4* __restrict__ w0,
                                           const float4* __restrict__ w1, int64_t n4,
                                           const float4* x4, int lane, float& a0, float& a1,
                                           int64_t s0 = 0, int64_t s1 = -1) {
    const int64_t full = n4 / kGemvStep;
    if (s1 < 0) s1 = full + 1;
    const int64_t send = s1 < full ? s1 : full;
    const float4* p0 = w0 + s0 * kGemvStep + lane;
    const float4* p1 = w1 + s0 * kGemvStep + lane;
    const float4* xp = x4 + s0 * kGemvStep + lane;
    for (int64_t s = s0; s < send; ++s) {
        float4 r0[4], r1[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            r0[u] = __ldcs(p0 + 32 * u);
            r1[u] = __ldcs(p1 + 32 * u);
        }
        p0 += kGemvStep;
        p1 += kGemvStep;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const float4 xv = ldx<XS>(xp + 32 * u);
            a0 = __fmaf_rn(xv.x, r0[u].x, a0);
            a0 = __fmaf_rn(xv.y, r0[u].y, a0);
            a0 = __fmaf_rn(xv.z, r0[u].z, a0);
            a0 = __fmaf_rn(xv.w, r0[u].w, a0);
            a1 = __fmaf_rn(xv.x, r1[u].x, a1);
            a1 = __fmaf_rn(xv.y, r1[u].y, a1);
            a1 = __fmaf_rn(xv.z, r1[u].z, a1);
            a1 = __fmaf_rn(xv.w, r1[u].w, a1);
        }
        xp += kGemvStep;
    }
    if (s1 <= full) return;
    for (int u = 0; u < 4; ++u) {
        const int64_t v = full * kGemvStep + 32 * u + lane;
        if (v >= n4) break;
        const float4 xv = ldx<XS>(x4 + v), r0 = __ldcs(w0 + v), r1 = __ldcs(w1 + v);
        a0 = __fmaf_rn(xv.x, r0.x, a0);
        a0 = __fmaf_rn(xv.y, r0.y, a0);
        a0 = __fmaf_rn(xv.z, r0.z, a0);
        a0 = __fmaf_rn(xv.w, r0.w, a0);
        a1 = __fmaf_rn(xv.x, r1.x, a1);
        a1 = __fmaf_rn(xv.y, r1.y, a1);
        a1 = __fmaf_rn(xv.z, r1.z, a1);
        a1 = __fmaf_rn(xv.w, r1.w, a1);
    }
}

// ------------------------------------------------------------- INT8 / INT4
// Quantized rows in the .tbm layout (Model::get_weight_fp32,
// include/tensorbit/run/model.hpp:181-225): element i of the tensor is byte
// i (INT8) or the low (even i) / high (odd i) nibble of byte i / 2 (INT4),
// two's complement, with an f32 scale per group of gs consecutive elements
// (1.0 past the last scale; the runner sends tensors with fewer scales than
// groups to the dequantising path).  The weight is (float)q * scale -- here
// too, so each product is the reference's; only the summation order differs.
//
// Lanes take consecutive 32-bit words (4 INT8 or 8 INT4 weights), so their
// float4s of x are contiguous across the warp; eight words per lane and row
// in flight.  q becomes a float without a conversion instruction: with its
// sign bit flipped it is an unsigned value u = q + 128 (or + 8), placed in
// the low mantissa bits of 2^23; subtracting 2^23 + 128 (or + 8) leaves q.
constexpr int kQU = 8;                  // words per lane per step
constexpr int kQStep = 32 * kQU;        // words per warp step

template <int BITS>
__device__ __forceinline__ float qval(uint32_t wx, int k) {  // wx: word with sign bits flipped
    if constexpr (BITS == 8)
        return __fsub_rn(__uint_as_float(__byte_perm(wx, 0x4B000000u, 0x7540u | (uint32_t)k)),
                         8388736.0f);
    else
        return __fsub_rn(__uint_as_float(0x4B000000u | ((wx >> (4 * k)) & 0xFu)), 8388616.0f);
}

// The scale of element f: the caller guarantees every group has one (a
// tensor of one group has gshift 31).
__device__ __forceinline__ float qscale(const float* sc, int gshift, uint32_t f) {
    return __ldg(sc + (f >> gshift));
}

// One word of a row against x: acc += x[e] * ((float)q[e] * scale).
// INT4: nibble k (k <= 4) enters the float in place, as 16^k (q + 8) in the
// low mantissa of 2^23, with no shift; subtracting 2^23 + 8 * 16^k leaves
// 16^k q, scaled by scale / 16^k (exact: a power of two), so the product is
// (float)q * scale.  Nibbles 5-7 are the same after one 16-bit shift.
template <int BITS, bool XS>
__device__ __forceinline__ float qword_dot(uint32_t w, float scale, const float4* x4, int64_t word,
                                           float acc) {
    if constexpr (BITS == 8) {
        const uint32_t wx = w ^ 0x80808080u;
        const float4 xv = ldx<XS>(x4 + word);
        acc = __fmaf_rn(xv.x, __fmul_rn(qval<8>(wx, 0), scale), acc);
        acc = __fmaf_rn(xv.y, __fmul_rn(qval<8>(wx, 1), scale), acc);
        acc = __fmaf_rn(xv.z, __fmul_rn(qval<8>(wx, 2), scale), acc);
        acc = __fmaf_rn(xv.w, __fmul_rn(qval<8>(wx, 3), scale), acc);
    } else {
        const uint32_t wx = w ^ 0x88888888u, hi = wx >> 16;
        const float s1 = __fmul_rn(scale, 0.0625f), s2 = __fmul_rn(scale, 0.00390625f);
        const float s3 = __fmul_rn(scale, 0.000244140625f), s4 = __fmul_rn(scale, 1.52587890625e-05f);
        const float4 xa = ldx<XS>(x4 + 2 * word), xb = ldx<XS>(x4 + 2 * word + 1);
        const float q0 = __fsub_rn(__uint_as_float((wx & 0xFu) | 0x4B000000u), 8388616.0f);
        const float q1 = __fsub_rn(__uint_as_float((wx & 0xF0u) | 0x4B000000u), 8388736.0f);
        const float q2 = __fsub_rn(__uint_as_float((wx & 0xF00u) | 0x4B000000u), 8390656.0f);
        const float q3 = __fsub_rn(__uint_as_float((wx & 0xF000u) | 0x4B000000u), 8421376.0f);
        const float q4 = __fsub_rn(__uint_as_float((wx & 0xF0000u) | 0x4B000000u), 8912896.0f);
        const float q5 = __fsub_rn(__uint_as_float((hi & 0xF0u) | 0x4B000000u), 8388736.0f);
        const float q6 = __fsub_rn(__uint_as_float((hi & 0xF00u) | 0x4B000000u), 8390656.0f);
        const float q7 = __fsub_rn(__uint_as_float((hi & 0xF000u) | 0x4B000000u), 8421376.0f);
        acc = __fmaf_rn(xa.x, __fmul_rn(q0, scale), acc);
        acc = __fmaf_rn(xa.y, __fmul_rn(q1, s1), acc);
        acc = __fmaf_rn(xa.z, __fmul_rn(q2, s2), acc);
        acc = __fmaf_rn(xa.w, __fmul_rn(q3, s3), acc);
        acc = __fmaf_rn(xb.x, __fmul_rn(q4, s4), acc);
        acc = __fmaf_rn(xb.y, __fmul_rn(q5, s1), acc);
        acc = __fmaf_rn(xb.z, __fmul_rn(q6, s2), acc);
        acc = __fmaf_rn(xb.w, __fmul_rn(q7, s3), acc);
    }
    return acc;
}

// A quantized row's scales: the tensor's scale array, log2 of its group
// size, and the flat index of the row's first element in the tensor.
struct QRow {
    const float* sc;  // one scale per group, every group present
    int gshift;       // 31 for a tensor of one group
    uint32_t f;       // tensors of fewer than 2^31 weights
};

// Partial sums of two quantized rows (which may belong to different
// tensors).  d0/d1: the rows' first words; words: words per row; steps
// [s0, s1) of kQStep words (all by default; the partial last step goes to
// whoever owns step words / kQStep).
template <int BITS, bool XS = false>
__device__ __forceinline__ void quant_dot2(const uint32_t* __restrict__ d0,
                                           const uint32_t* __restrict__ d1, const QRow q0,
                                           const QRow q1, int64_t words, const float4* x4,
                                           int lane, float& a0, float& a1, int64_t s0 = 0,
                                           int64_t s1 = -1) {
    constexpr int kPer = 32 / BITS;
    const int64_t full = words / kQStep;
    if (s1 < 0) s1 = full + 1;
    const int64_t send = s1 < full ? s1 : full;
    for (int64_t s = s0; s < send; ++s) {
        const int64_t w0 = s * kQStep + lane;
        uint32_t r0[kQU], r1[kQU];
#pragma unroll
        for (int u = 0; u < kQU; ++u) {
            r0[u] = __ldcs(d0 + w0 + 32 * u);
            r1[u] = __ldcs(d1 + w0 + 32 * u);
        }
#pragma unroll
        for (int u = 0; u < kQU; ++u) {
            const int64_t w = w0 + 32 * u;
            const uint32_t e = (uint32_t)w * kPer;
            a0 = qword_dot<BITS, XS>(r0[u], qscale(q0.sc, q0.gshift, q0.f + e), x4, w,
                                     a0);
            a1 = qword_dot<BITS, XS>(r1[u], qscale(q1.sc, q1.gshift, q1.f + e), x4, w,
                                     a1);
        }
    }
    if (s1 <= full) return;
    for (int u = 0; u < kQU; ++u) {  // the partial step
        const int64_t w = full * kQStep + 32 * u + lane;
        if (w >= words) break;
        const uint32_t e = (uint32_t)w * kPer;
        a0 = qword_dot<BITS, XS>(__ldcs(d0 + w), qscale(q0.sc, q0.gshift, q0.f + e),
                                 x4, w, a0);
        a1 = qword_dot<BITS, XS>(__ldcs(d1 + w), qscale(q1.sc, q1.gshift, q1.f + e),
                                 x4, w, a1);
    }
}

__device__ __forceinline__ void warp_sum2(float& a0, float& a1) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        a0 = __fadd_rn(a0, __shfl_xor_sync(kFull, a0, o));
        a1 = __fadd_rn(a1, __shfl_xor_sync(kFull, a1, o));
    }
}

}  // namespace tbk
