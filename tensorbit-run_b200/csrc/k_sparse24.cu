// k_sparse24.cu -- 2:4 sparse weights packed to their kept values, and the
// GEMV over that packed form.
//
// The reference stores an N:M-pruned layer dense (pruned weights 0) with one
// mask byte per group of four columns, and its sparse GEMV reads all of it
// (src/ops/linear.c:4-35): 4.25 bytes per weight.  A true 2:4 layer keeps at
// most two weights per group, so the device keeps only those: per pair of
// groups one float4 of values (kept weights in column order, 0 in an unused
// slot) and one index byte (2 bits per slot: the column within its group).
// That is 2.125 bytes per weight, half the traffic, for the same sum of
// x[col] * w[col] over the kept columns -- added in a different order from
// the reference's left-to-right loop, so results agree within the f32 row
// tolerance, as the dense-layout kernel's do.
//
// Packing runs once (a model load); a group with three or four mask bits set
// cannot be packed and is reported, so the caller keeps the dense layout.
// The GEMV gives each warp two output rows, so each float4 of x loaded
// through L1 serves both; lanes take consecutive group pairs, four in flight.
#include "tb_device.cuh"
#include "tb_internal.h"

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kU = 4;  // group pairs in flight per lane and row

// Pack pair p of row j: groups 2p and 2p+1 (columns 8p .. 8p+7).
__global__ void __launch_bounds__(kThreads)
k_pack24(int64_t rows, int64_t groups, int64_t in_f, const float* __restrict__ w,
         const uint8_t* __restrict__ mask, float4* __restrict__ vals, uint8_t* __restrict__ idx,
         int* __restrict__ unpackable) {
    const int64_t pairs = (groups + 1) / 2;
    const int64_t total = rows * pairs;
    for (int64_t t = (int64_t)blockIdx.x * kThreads + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * kThreads) {
        const int64_t j = t / pairs, p = t - j * pairs;
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        uint32_t ib = 0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int64_t g = 2 * p + h;
            if (g >= groups) break;
            const uint32_t m = mask[j * groups + g] & 0xFu;  // bits k < 4 (linear.c:22-23)
            const float* wr = w + j * in_f + 4 * g;
            int slot = 0, first = 0;
            for (int k = 0; k < 4; ++k) {
                if (!(m & (1u << k))) continue;
                if (slot == 2) {
                    atomicExch(unpackable, 1);
                    break;
                }
                if (slot == 0) first = k;
                v[2 * h + slot] = wr[k];
                ib |= (uint32_t)k << (4 * h + 2 * slot);
                ++slot;
            }
            if (slot == 1) ib |= (uint32_t)first << (4 * h + 2);  // unused slot: value 0
        }
        vals[t] = make_float4(v[0], v[1], v[2], v[3]);
        idx[t] = (uint8_t)ib;
    }
}

__device__ __forceinline__ float pick(const float4& x, uint32_t k) {
    return k == 0 ? x.x : k == 1 ? x.y : k == 2 ? x.z : x.w;
}

__device__ __forceinline__ float pair_dot(const float4& v, uint32_t ib, const float4& xa,
                                          const float4& xb, float acc) {
    acc = __fmaf_rn(v.x, pick(xa, ib & 3u), acc);
    acc = __fmaf_rn(v.y, pick(xa, (ib >> 2) & 3u), acc);
    acc = __fmaf_rn(v.z, pick(xb, (ib >> 4) & 3u), acc);
    acc = __fmaf_rn(v.w, pick(xb, ib >> 6), acc);
    return acc;
}

// Two output rows per warp; `pairs` group pairs per row (groups even).
__global__ void __launch_bounds__(kThreads)
k_linear24(int64_t rows, int64_t pairs, const float* __restrict__ x,
           const float4* __restrict__ vals, const uint8_t* __restrict__ idx,
           const float* bias, float* y) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * kWarps;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    for (int64_t j0 = 2 * ((int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5)); j0 < rows;
         j0 += 2 * warps) {
        const bool two = j0 + 1 < rows;
        const float4* v0 = vals + j0 * pairs;
        const float4* v1 = two ? v0 + pairs : v0;
        const uint8_t* i0 = idx + j0 * pairs;
        const uint8_t* i1 = two ? i0 + pairs : i0;
        float a0 = 0.0f, a1 = 0.0f;
        for (int64_t p0 = lane; p0 < pairs; p0 += 32 * kU) {
            float4 w0[kU], w1[kU];
            uint32_t b0[kU], b1[kU];
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int64_t p = p0 + 32 * u;
                const bool in = p < pairs;
                w0[u] = in ? __ldcs(v0 + p) : make_float4(0.f, 0.f, 0.f, 0.f);
                w1[u] = in ? __ldcs(v1 + p) : make_float4(0.f, 0.f, 0.f, 0.f);
                b0[u] = in ? (uint32_t)__ldcs(i0 + p) : 0u;
                b1[u] = in ? (uint32_t)__ldcs(i1 + p) : 0u;
            }
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int64_t p = p0 + 32 * u;
                if (p >= pairs) break;
                const float4 xa = __ldg(x4 + 2 * p), xb = __ldg(x4 + 2 * p + 1);
                a0 = pair_dot(w0[u], b0[u], xa, xb, a0);
                a1 = pair_dot(w1[u], b1[u], xa, xb, a1);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            a0 = __fadd_rn(a0, __shfl_xor_sync(tbk::kFull, a0, o));
            a1 = __fadd_rn(a1, __shfl_xor_sync(tbk::kFull, a1, o));
        }
        if (lane == 0) {
            y[j0] = bias ? __fadd_rn(bias[j0], a0) : a0;
            if (two) y[j0 + 1] = bias ? __fadd_rn(bias[j0 + 1], a1) : a1;
        }
    }
}

}  // namespace

extern "C" int tb_b200_sparse24_pack(int64_t out_features, int64_t in_features, const float* w,
                                     const uint8_t* mask, void* vals, uint8_t* idx,
                                     int* unpackable_dev, void* stream) {
    if (out_features < 0 || in_features < 0) return TB_ERR_INVALID_SHAPE;
    if (!w || !mask || !vals || !idx || !unpackable_dev) return TB_ERR_INVALID_ARG;
    const int64_t groups = in_features / 4;
    const int64_t pairs = (groups + 1) / 2;
    if (out_features == 0 || pairs == 0) return TB_OK;
    if (!tbh::aligned16(vals)) return TB_ERR_INVALID_ARG;
    const tbh::DeviceState* ds = tbh::current_device_state();
    if (!ds) return TB_ERR_DEVICE;
    cudaStream_t s = tbh::stream_of(stream);
    k_pack24<<<tbh::ew_grid(out_features * pairs, kThreads, ds), kThreads, 0, s>>>(
        out_features, groups, in_features, w, mask, static_cast<float4*>(vals), idx,
        unpackable_dev);
    TB_LAUNCH_CHECK("2:4 pack kernel");
    return TB_OK;
}

extern "C" int tb_b200_sparse24_linear(int64_t out_features, int64_t in_features, const float* x,
                                       const void* vals, const uint8_t* idx, const float* bias,
                                       float* y, void* stream) {
    if (out_features < 0 || in_features < 0) return TB_ERR_INVALID_SHAPE;
    if (!x || !vals || !idx || !y) return TB_ERR_INVALID_ARG;
    if (out_features == 0) return TB_OK;
    const int64_t groups = in_features / 4;
    if (groups % 2) return TB_ERR_INVALID_SHAPE;  // whole pairs: in_features / 4 even
    if (!tbh::aligned16(x) || !tbh::aligned16(vals)) return TB_ERR_INVALID_ARG;
    const tbh::DeviceState* ds = tbh::current_device_state();
    if (!ds) return TB_ERR_DEVICE;
    cudaStream_t s = tbh::stream_of(stream);
    if (groups == 0) {  // no used columns: y = bias or 0
        if (bias)
            TB_CUDA_TRY(cudaMemcpyAsync(y, bias, (size_t)out_features * 4, cudaMemcpyDeviceToDevice, s));
        else
            TB_CUDA_TRY(cudaMemsetAsync(y, 0, (size_t)out_features * 4, s));
        return TB_OK;
    }
    const int grid = tbh::ew_grid((out_features + 1) / 2, kWarps, ds, 16);
    k_linear24<<<grid, kThreads, 0, s>>>(out_features, groups / 2, x,
                                         static_cast<const float4*>(vals), idx, bias, y);
    TB_LAUNCH_CHECK("2:4 packed linear kernel");
    return TB_OK;
}
