// bodies.cuh -- per-CTA bodies of the row kernels, written against a
// "virtual block" index so the standalone kernels (one body per launch) and
// the fused layer-chain kernel (three bodies in one launch, partitioned by
// block range) share one implementation and give identical bits.
//
// Reference arithmetic of each body is stated where it is defined; every
// operation uses an explicit round-to-nearest intrinsic so the rounding is
// the reference Release build's: FMA only where gcc contracted there (the
// RMSNorm sum of squares, GELU's v + 0.044715*v^3), separate roundings
// everywhere else.
#pragma once

#include <math.h>

#include "tb_device.cuh"

namespace tbk {

// ============================================================ RMSNorm
// residual add + RMSNorm (src/ops/residual.c:4-13, src/ops/norm.c:4-26):
//   h = x + residual;  scale = 1/sqrtf((eps + sum h^2)/cols);  y = (h*scale)*w
// The sum of squares is a per-thread FMA chain, a warp tree and then the
// warps in order (the CPU's is one left-to-right FMA chain): `scale` may
// differ by a few ulp, nothing else does.
//
// A row belongs to G threads (G a power of two, 32..1024, G <= blockDim);
// thread `lane` of the group owns vectors lane, lane+G, ... (ITEMS at most),
// loads all of them before any arithmetic and keeps h in registers.
// Aliasing: y/h_out may be the same buffers as x/residual (every element is
// read before it is written, by the thread that writes it).
template <typename T, int VEC, int ITEMS>
__device__ __forceinline__ void res_rms_body(const T* x, const T* res, const T* w, T* h_out, T* y,
                                             int64_t rows, int cols, float eps, int G,
                                             int64_t vblock, float* red) {
    // Raw 16-byte vectors are kept (half the registers of f32 copies for
    // bf16) and h = x + residual is recomputed after the reduction: the same
    // single f32 add, so the same bits.
    using Raw = typename Elt<T>::template Raw<VEC>;
    const int lane = threadIdx.x & (G - 1);
    const int64_t row = vblock * (blockDim.x / G) + threadIdx.x / G;
    const bool active = row < rows;
    const int nvec = cols / VEC;
    const int64_t base = row * (int64_t)cols;

    Raw rx[ITEMS], rr[ITEMS];
    if (active) {
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) {
            const int vi = lane + i * G;
            if (vi < nvec) {
                rx[i] = Elt<T>::template load_raw<VEC>(x + base + (int64_t)vi * VEC);
                if (res != nullptr) rr[i] = Elt<T>::template load_raw<VEC>(res + base + (int64_t)vi * VEC);
            }
        }
    }
    float ss = 0.0f;
    if (active) {
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) {
            if (lane + i * G < nvec) {
                float h[VEC];
                Elt<T>::template widen<VEC>(rx[i], h);
                if (res != nullptr) {
                    float r[VEC];
                    Elt<T>::template widen<VEC>(rr[i], r);
#pragma unroll
                    for (int j = 0; j < VEC; ++j) h[j] = __fadd_rn(h[j], r[j]);
                }
#pragma unroll
                for (int j = 0; j < VEC; ++j) ss = __fmaf_rn(h[j], h[j], ss);
            }
        }
    }
    ss = group_sum(ss, G, red);
    if (!active) return;
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(__fadd_rn(ss, eps), (float)cols)));
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
        const int vi = lane + i * G;
        if (vi >= nvec) continue;
        const int64_t off = base + (int64_t)vi * VEC;
        float h[VEC];
        Elt<T>::template widen<VEC>(rx[i], h);
        if (res != nullptr) {
            float r[VEC];
            Elt<T>::template widen<VEC>(rr[i], r);
#pragma unroll
            for (int j = 0; j < VEC; ++j) h[j] = __fadd_rn(h[j], r[j]);
        }
        if (h_out != nullptr) store_vec<T, VEC>(h_out + off, h);
        float o[VEC];
        if (w != nullptr) {
            float g[VEC];
            load_vec<T, VEC>(w + (int64_t)vi * VEC, g);
#pragma unroll
            for (int j = 0; j < VEC; ++j) o[j] = __fmul_rn(__fmul_rn(h[j], scale), g[j]);
        } else {
#pragma unroll
            for (int j = 0; j < VEC; ++j) o[j] = __fmul_rn(h[j], scale);
        }
        store_vec<T, VEC>(y + off, o);
    }
}

// ============================================================ RoPE
// Interleaved-pair rotation (tb_cpu_rope_gqa_f32, src/ops/rope.c:43-81):
//   (a0, a1) -> (a0*c - a1*s, a1*c + a0*s), every product rounded.
constexpr int kRopeMaxPairs = 256;  // head_dim <= 512

struct RopeConst {
    float inv_freq[kRopeMaxPairs];  // f_i = 1.0f/powf(theta, 2i/d), host C library
    float2 cs[kRopeMaxPairs];       // single-position mode: (cos, sin) per pair
};

enum RopeMode { kRopePerRow = 0, kRopeConst = 1 };

__device__ __forceinline__ void rope_rotate(float& a0, float& a1, float c, float s) {
    const float r0 = __fsub_rn(__fmul_rn(a0, c), __fmul_rn(a1, s));
    const float r1 = __fadd_rn(__fmul_rn(a1, c), __fmul_rn(a0, s));
    a0 = r0;
    a1 = r1;
}

// One token row: q row [hq, d], k row [hkv, d], in place.  A thread owns
// VEC consecutive elements (VEC/2 pairs) of a head, so its cos/sin are
// fetched once and reused for every head; UNROLL heads are loaded before
// any is rotated.  cos/sin: the host-built table (bit-identical to the
// reference) for positions in [0, table_pos), else device sincosf of the
// same f32 angle (pos * f_i).
template <typename T, int VEC, int MODE, int UNROLL>
__device__ __forceinline__ void rope_body(T* q, T* k, const int32_t* positions, int hq, int hkv,
                                          int d, const float2* table, int table_pos,
                                          const RopeConst& rc, int64_t row) {
    constexpr int P = VEC / 2;
    const int lanes = d / VEC;
    const int j = threadIdx.x % lanes;
    const int h0 = threadIdx.x / lanes;
    const int hstep = blockDim.x / lanes;
    if (h0 >= hstep) return;
    const int nh = hq + hkv;

    T* qrow = q + row * (int64_t)hq * d;
    T* krow = k + row * (int64_t)hkv * d;
    // The head loads do not depend on the position: issue the first batch
    // before the position -> table chain.  Heads stay in their raw 16-byte
    // form until they are rotated (few registers, more CTAs per SM).
    using Raw = typename Elt<T>::template Raw<VEC>;
    Raw v[UNROLL];
    T* ptr[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
        const int h = h0 + u * hstep;
        ptr[u] = nullptr;
        if (h < nh) {
            ptr[u] = (h < hq ? qrow + (int64_t)h * d : krow + (int64_t)(h - hq) * d) + j * VEC;
            v[u] = Elt<T>::template load_raw_keep<VEC>(ptr[u]);
        }
    }
    float c[P], s[P];
    if constexpr (MODE == kRopeConst) {
#pragma unroll
        for (int p = 0; p < P; ++p) {
            c[p] = rc.cs[j * P + p].x;
            s[p] = rc.cs[j * P + p].y;
        }
    } else {
        const int pos = positions[row];
        if (table != nullptr && pos >= 0 && pos < table_pos) {
            const float2* t = table + (int64_t)pos * (d / 2) + j * P;
#pragma unroll
            for (int p = 0; p < P; ++p) {
                const float2 cv = t[p];
                c[p] = cv.x;
                s[p] = cv.y;
            }
        } else {
#pragma unroll
            for (int p = 0; p < P; ++p) {
                const float ang = __fmul_rn((float)pos, rc.inv_freq[j * P + p]);
                sincosf(ang, &s[p], &c[p]);
            }
        }
    }

    for (int hb = h0; hb < nh; hb += UNROLL * hstep) {
        if (hb != h0) {
#pragma unroll
            for (int u = 0; u < UNROLL; ++u) {
                const int h = hb + u * hstep;
                ptr[u] = nullptr;
                if (h < nh) {
                    ptr[u] = (h < hq ? qrow + (int64_t)h * d : krow + (int64_t)(h - hq) * d) + j * VEC;
                    v[u] = Elt<T>::template load_raw_keep<VEC>(ptr[u]);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            if (ptr[u] == nullptr) continue;
            float f[VEC];
            Elt<T>::template widen<VEC>(v[u], f);
#pragma unroll
            for (int p = 0; p < P; ++p) rope_rotate(f[2 * p], f[2 * p + 1], c[p], s[p]);
            store_vec<T, VEC>(ptr[u], f);
        }
    }
}

// ============================================================ elementwise
//   silu(v)  = v / (1 + expf(-v))                        src/ops/activation.c:18-27
//   gelu(v)  = (0.5*v) * (1 + tanhf(k*fma(0.044715, (v*v)*v, v)))
//                                                       src/ops/activation.c:4-16
//   swiglu   = silu(gate) * up                           include/tensorbit/run/ops.hpp:246-248
//   add      = x + residual                              src/ops/residual.c:4-13
// expf/tanhf: CUDA's full-precision functions (within 2 ulp of the C
// library's); '/' is the IEEE division.
enum EwOp { kSilu = 0, kGelu = 1, kSwiglu = 2, kAdd = 3 };

constexpr float kSqrt2OverPi = 0.79788456080286535588f;

__device__ __forceinline__ float silu_f(float v) { return __fdiv_rn(v, __fadd_rn(1.0f, expf(-v))); }

__device__ __forceinline__ float gelu_f(float v) {
    const float cube = __fmul_rn(__fmul_rn(v, v), v);
    const float arg = __fmul_rn(kSqrt2OverPi, __fmaf_rn(0.044715f, cube, v));
    return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, tanhf(arg)));
}

template <int OP>
__device__ __forceinline__ float ew_apply(float a, float b) {
    if constexpr (OP == kSilu) return silu_f(a);
    if constexpr (OP == kGelu) return gelu_f(a);
    if constexpr (OP == kSwiglu) return __fmul_rn(silu_f(a), b);
    return __fadd_rn(a, b);
}

template <int OP>
constexpr bool ew_binary() {
    return OP == kSwiglu || OP == kAdd;
}

// Grid-stride over nvec vectors as virtual block `vblock` of `vgrid`.
// UNROLL > 1: UNROLL vectors per thread per round, all loads first (cheap
// ops).  UNROLL == 1: the next vector's load is issued before the current
// one is computed, and vectors stay in their raw 16-byte form until then
// (transcendental ops: few registers, two loads in flight per thread).
template <typename T, int VEC, int OP, int UNROLL>
__device__ __forceinline__ void ew_body(const T* a, const T* b, T* out, int64_t nvec,
                                        int64_t vblock, int64_t vgrid) {
    const int64_t stride = vgrid * blockDim.x;
    int64_t i = vblock * blockDim.x + threadIdx.x;
    if constexpr (UNROLL == 1) {
        using Raw = typename Elt<T>::template Raw<VEC>;
        if (i >= nvec) return;
        Raw na = Elt<T>::template load_raw<VEC>(a + i * VEC), nb;
        if constexpr (ew_binary<OP>()) nb = Elt<T>::template load_raw<VEC>(b + i * VEC);
        for (; i < nvec; i += stride) {
            const Raw ca = na;
            Raw cb;
            if constexpr (ew_binary<OP>()) cb = nb;
            const int64_t n = i + stride;
            if (n < nvec) {
                na = Elt<T>::template load_raw<VEC>(a + n * VEC);
                if constexpr (ew_binary<OP>()) nb = Elt<T>::template load_raw<VEC>(b + n * VEC);
            }
            float va[VEC], vb[VEC], o[VEC];
            Elt<T>::template widen<VEC>(ca, va);
            if constexpr (ew_binary<OP>()) Elt<T>::template widen<VEC>(cb, vb);
#pragma unroll
            for (int j = 0; j < VEC; ++j) o[j] = ew_apply<OP>(va[j], ew_binary<OP>() ? vb[j] : 0.0f);
            store_vec<T, VEC>(out + i * VEC, o);
        }
    } else {
    for (; i + (UNROLL - 1) * stride < nvec; i += UNROLL * stride) {
        float va[UNROLL][VEC], vb[UNROLL][VEC];
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            load_vec_stream<T, VEC>(a + (i + u * stride) * VEC, va[u]);
            if constexpr (ew_binary<OP>()) load_vec_stream<T, VEC>(b + (i + u * stride) * VEC, vb[u]);
        }
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            float o[VEC];
#pragma unroll
            for (int j = 0; j < VEC; ++j) o[j] = ew_apply<OP>(va[u][j], ew_binary<OP>() ? vb[u][j] : 0.0f);
            store_vec<T, VEC>(out + (i + u * stride) * VEC, o);
        }
    }
    for (; i < nvec; i += stride) {
        float va[VEC], vb[VEC], o[VEC];
        load_vec_stream<T, VEC>(a + i * VEC, va);
        if constexpr (ew_binary<OP>()) load_vec_stream<T, VEC>(b + i * VEC, vb);
#pragma unroll
        for (int j = 0; j < VEC; ++j) o[j] = ew_apply<OP>(va[j], ew_binary<OP>() ? vb[j] : 0.0f);
        store_vec<T, VEC>(out + i * VEC, o);
    }
    }
}

}  // namespace tbk
