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
// The GEMV is tbk::packed_dot2 (gemv.cuh): two output rows per warp, so each
// float4 of x loaded through L1 serves both, four pairs per lane and row in
// flight, the index bytes laid out so each lane loads its four as one word.
#include "gemv.cuh"
#include "tb_internal.h"

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

// Pack pair p of row j: groups 2p and 2p+1 (columns 8p .. 8p+7).
__global__ void __launch_bounds__(kThreads)
k_pack24(int64_t rows, int64_t groups, int64_t in_f, const float* __restrict__ w,
         const uint8_t* __restrict__ mask, float4* __restrict__ vals, uint8_t* __restrict__ idx,
         int* __restrict__ unpackable) {
    const int64_t pairs = (groups + 1) / 2;
    const int64_t istride = tbk::packed_idx_stride(pairs);
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
        const int64_t r = p % tbk::kGemvStep;  // byte of pair p: 128 s + 4 l + u
        idx[j * istride + (p - r) + 4 * (r % 32) + r / 32] = (uint8_t)ib;
    }
}

// Two output rows per warp (the same row twice for an odd last row).
__global__ void __launch_bounds__(kThreads)
k_linear24(int64_t rows, int64_t pairs, int64_t istride, const float* __restrict__ x,
           const float4* __restrict__ vals, const uint8_t* __restrict__ idx, const float* bias,
           float* y) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * kWarps;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    for (int64_t j0 = 2 * ((int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5)); j0 < rows;
         j0 += 2 * warps) {
        const int64_t j1 = j0 + 1 < rows ? j0 + 1 : j0;
        float a0 = 0.0f, a1 = 0.0f;
        tbk::packed_dot2(vals + j0 * pairs, idx + j0 * istride, vals + j1 * pairs,
                         idx + j1 * istride, pairs, x4, lane, a0, a1);
        tbk::warp_sum2(a0, a1);
        if (lane == 0) {
            y[j0] = bias ? __fadd_rn(bias[j0], a0) : a0;
            if (j1 != j0) y[j1] = bias ? __fadd_rn(bias[j1], a1) : a1;
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
    if (!tbh::aligned16(x) || !tbh::aligned16(vals) || reinterpret_cast<uintptr_t>(idx) % 4)
        return TB_ERR_INVALID_ARG;
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
    k_linear24<<<grid, kThreads, 0, s>>>(out_features, groups / 2,
                                         tbk::packed_idx_stride(groups / 2), x,
                                         static_cast<const float4*>(vals), idx, bias, y);
    TB_LAUNCH_CHECK("2:4 packed linear kernel");
    return TB_OK;
}
