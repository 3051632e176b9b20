// tb_device.cuh -- device-side helpers shared by the sm_100a row kernels:
// 16-byte vector access for f32/bf16 rows, exact-rounding arithmetic
// wrappers, and warp/group reductions.
//
// Every row kernel in this library is HBM-bandwidth bound (< 2 flop/byte),
// so the helpers are about moving bytes: one 16-byte load or store per
// access (4 f32 or 8 bf16), issued before any arithmetic so each thread keeps
// several in flight.  Arithmetic uses the explicit round-to-nearest
// intrinsics (__fadd_rn, __fmul_rn, __fmaf_rn, __fdiv_rn, __fsqrt_rn) so the
// compiler can neither contract nor reassociate: each kernel states exactly
// which operations fuse, matching how the reference C build rounds.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

namespace tbk {

constexpr unsigned kFull = 0xffffffffu;

// ---------------------------------------------------------------- elements
template <typename T>
struct Elt;

// Raw<VEC>: VEC elements kept in their storage format (one 16-byte word
// for a full vector); load_raw streams them in (evict-first), widen turns
// them into f32.
template <typename T, int VEC>
struct RawOf {
    T e[VEC];
};

template <>
struct Elt<float> {
    static constexpr int kVec = 4;  // elements per 16-byte access
    template <int VEC>
    using Raw = typename std::conditional<VEC == 4, uint4, RawOf<float, VEC>>::type;
    __device__ __forceinline__ static float load(const float* p) { return *p; }
    __device__ __forceinline__ static void store(float* p, float v) { *p = v; }
    template <int VEC>
    __device__ __forceinline__ static Raw<VEC> load_raw(const float* p) {
        if constexpr (VEC == 4) {
            return __ldcs(reinterpret_cast<const uint4*>(p));
        } else {
            Raw<VEC> r;
#pragma unroll
            for (int i = 0; i < VEC; ++i) r.e[i] = p[i];
            return r;
        }
    }
    // Same, with the default caching (the data is read again or written back).
    template <int VEC>
    __device__ __forceinline__ static Raw<VEC> load_raw_keep(const float* p) {
        if constexpr (VEC == 4) {
            return *reinterpret_cast<const uint4*>(p);
        } else {
            Raw<VEC> r;
#pragma unroll
            for (int i = 0; i < VEC; ++i) r.e[i] = p[i];
            return r;
        }
    }
    template <int VEC>
    __device__ __forceinline__ static void widen(const Raw<VEC>& r, float (&v)[VEC]) {
        if constexpr (VEC == 4) {
            v[0] = __uint_as_float(r.x); v[1] = __uint_as_float(r.y);
            v[2] = __uint_as_float(r.z); v[3] = __uint_as_float(r.w);
        } else {
#pragma unroll
            for (int i = 0; i < VEC; ++i) v[i] = r.e[i];
        }
    }
};

template <>
struct Elt<__nv_bfloat16> {
    static constexpr int kVec = 8;
    template <int VEC>
    using Raw = typename std::conditional<VEC == 8, uint4, RawOf<__nv_bfloat16, VEC>>::type;
    __device__ __forceinline__ static float load(const __nv_bfloat16* p) {
        return __bfloat162float(*p);
    }
    __device__ __forceinline__ static void store(__nv_bfloat16* p, float v) {
        *p = __float2bfloat16_rn(v);
    }
    template <int VEC>
    __device__ __forceinline__ static Raw<VEC> load_raw(const __nv_bfloat16* p) {
        if constexpr (VEC == 8) {
            return __ldcs(reinterpret_cast<const uint4*>(p));
        } else {
            Raw<VEC> r;
#pragma unroll
            for (int i = 0; i < VEC; ++i) r.e[i] = p[i];
            return r;
        }
    }
    template <int VEC>
    __device__ __forceinline__ static Raw<VEC> load_raw_keep(const __nv_bfloat16* p) {
        if constexpr (VEC == 8) {
            return *reinterpret_cast<const uint4*>(p);
        } else {
            Raw<VEC> r;
#pragma unroll
            for (int i = 0; i < VEC; ++i) r.e[i] = p[i];
            return r;
        }
    }
    template <int VEC>
    __device__ __forceinline__ static void widen(const Raw<VEC>& r, float (&v)[VEC]) {
        if constexpr (VEC == 8) {
            const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                v[2 * i] = __uint_as_float(w[i] << 16);
                v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
            }
        } else {
#pragma unroll
            for (int i = 0; i < VEC; ++i) v[i] = __bfloat162float(r.e[i]);
        }
    }
};

// Load VEC consecutive elements starting at p (16-byte aligned when VEC is
// the full vector width) into f32 registers.
template <typename T, int VEC>
__device__ __forceinline__ void load_vec(const T* p, float (&v)[VEC]) {
    if constexpr (VEC == Elt<T>::kVec) {
        const uint4 raw = *reinterpret_cast<const uint4*>(p);
        if constexpr (sizeof(T) == 4) {
            v[0] = __uint_as_float(raw.x);
            v[1] = __uint_as_float(raw.y);
            v[2] = __uint_as_float(raw.z);
            v[3] = __uint_as_float(raw.w);
        } else {
            const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                v[2 * i] = __uint_as_float(w[i] << 16);
                v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < VEC; ++i) v[i] = Elt<T>::load(p + i);
    }
}

// Streaming variant for data read exactly once (evict-first in L1/L2).
template <typename T, int VEC>
__device__ __forceinline__ void load_vec_stream(const T* p, float (&v)[VEC]) {
    if constexpr (VEC == Elt<T>::kVec) {
        const uint4 raw = __ldcs(reinterpret_cast<const uint4*>(p));
        if constexpr (sizeof(T) == 4) {
            v[0] = __uint_as_float(raw.x);
            v[1] = __uint_as_float(raw.y);
            v[2] = __uint_as_float(raw.z);
            v[3] = __uint_as_float(raw.w);
        } else {
            const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                v[2 * i] = __uint_as_float(w[i] << 16);
                v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
            }
        }
    } else {
        load_vec<T, VEC>(p, v);
    }
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    const __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&b);
}

template <typename T, int VEC>
__device__ __forceinline__ void store_vec(T* p, const float (&v)[VEC]) {
    if constexpr (VEC == Elt<T>::kVec) {
        uint4 raw;
        if constexpr (sizeof(T) == 4) {
            raw = make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]),
                             __float_as_uint(v[3]));
        } else {
            raw = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                             pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
        }
        *reinterpret_cast<uint4*>(p) = raw;
    } else {
#pragma unroll
        for (int i = 0; i < VEC; ++i) Elt<T>::store(p + i, v[i]);
    }
}

// ---------------------------------------------------------------- reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(kFull, v, o));
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
    return v;
}

// Sum over a group of G threads (G a power of two, 32 <= G <= 1024) laid out
// contiguously in the block.  `red` is shared scratch of blockDim/32 floats.
// Every thread of the block must call it (it contains __syncthreads when
// G > 32).  Warp partials are combined in warp order, so the result is
// deterministic.
__device__ __forceinline__ float group_sum(float v, int G, float* red) {
    v = warp_sum(v);
    if (G <= 32) return v;
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) red[warp] = v;
    __syncthreads();
    const int first = (threadIdx.x / G) * (G >> 5);
    float s = red[first];
    for (int w = 1; w < (G >> 5); ++w) s = __fadd_rn(s, red[first + w]);
    __syncthreads();
    return s;
}

__device__ __forceinline__ float block_max(float v, float* red) {
    v = warp_max(v);
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if ((threadIdx.x & 31) == 0) red[warp] = v;
    __syncthreads();
    float m = red[0];
    for (int w = 1; w < nw; ++w) m = fmaxf(m, red[w]);
    __syncthreads();
    return m;
}

// ---------------------------------------------------------------- status
// Bits a kernel may raise in the per-device status word.
constexpr unsigned kFlagTokenRange = 0x1u;

}  // namespace tbk
