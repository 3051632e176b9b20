// k_dequant.cu -- INT4 / INT8 weights to f32 or bf16 on the device, bit-exact
// with the reference's dequantisation.
//
// Reference (tensorbit::run::Model::get_weight_fp32,
// include/tensorbit/run/model.hpp:181-225), over the n = rows * cols weights
// of a .tbm layer: element i is in scale group g = i / gs (gs = group_size,
// or n when it is 0); scale = scales[g] when g < the scale count, else 1;
// INT4 holds element i in the low nibble of byte i / 2 when i is even, the
// high nibble when odd, two's complement; INT8 is one signed byte.  The
// weight is (float)q * scale, one f32 multiply -- exactly this kernel's
// arithmetic, so f32 output is bit-identical and bf16 output is its
// round-to-nearest-even.
//
// HBM bound: n/2 (INT4) or n (INT8) bytes read, 4n or 2n written.  Consecutive
// lanes take consecutive chunks of 8 weights (4 or 8 bytes in, 16 or 32
// bytes out, so every warp access is one contiguous span), four chunks in
// flight per thread before any arithmetic; a chunk's scale group is one
// shift (power-of-two groups) or division, then stepped, never a division per
// weight; the grid strides over the tensor.  Unaligned buffers and the tail
// past the last chunk run one weight per thread.
#include <cuda_bf16.h>

#include "tb_device.cuh"
#include "tb_internal.h"

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ int nibble(uint32_t word, int k) {  // k-th 4-bit field, signed
    const int v = (int)((word >> (4 * k)) & 0xFu);
    return (v & 8) ? v - 16 : v;
}

__device__ __forceinline__ float scale_of(const float* scales, int64_t ns, int64_t g) {
    return g < ns ? scales[g] : 1.0f;
}

constexpr int kE = 8;      // weights per lane chunk: 4 (INT4) or 8 (INT8) bytes in
constexpr int kLoads = 4;  // chunks in flight per thread and step

__device__ __forceinline__ int64_t group_of(int64_t i, int64_t gs, int shift) {
    return shift >= 0 ? i >> shift : i / gs;
}

// Consecutive lanes take consecutive 8-weight chunks, so loads and stores of
// a warp instruction cover one contiguous span.
template <int SRC, typename OUT>
__global__ void __launch_bounds__(kThreads)
k_dequant_vec(const uint8_t* src, const float* scales, int64_t ns, int64_t gs, int shift,
              int64_t nchunks, OUT* dst) {
    const int64_t stride = (int64_t)gridDim.x * kThreads;
    for (int64_t c0 = (int64_t)blockIdx.x * kThreads + threadIdx.x; c0 < nchunks;
         c0 += stride * kLoads) {
        uint2 w[kLoads];
#pragma unroll
        for (int l = 0; l < kLoads; ++l) {
            const int64_t c = c0 + l * stride;
            w[l] = make_uint2(0u, 0u);
            if (c < nchunks) {
                if (SRC == TB_DTYPE_INT4)
                    w[l].x = __ldcs(reinterpret_cast<const unsigned int*>(src) + c);
                else
                    w[l] = __ldcs(reinterpret_cast<const uint2*>(src) + c);
            }
        }
#pragma unroll
        for (int l = 0; l < kLoads; ++l) {
            const int64_t c = c0 + l * stride;
            if (c >= nchunks) break;
            const int64_t i0 = c * kE;
            int64_t g = group_of(i0, gs, shift), b = (g + 1) * gs;
            float scale = scale_of(scales, ns, g);
            float o[kE];
#pragma unroll
            for (int k = 0; k < kE; ++k) {
                while (i0 + k >= b) {  // next scale group (several when gs < 8)
                    ++g;
                    b += gs;
                    scale = scale_of(scales, ns, g);
                }
                const int q = SRC == TB_DTYPE_INT4
                                  ? nibble(w[l].x, k)
                                  : (int)(int8_t)(((k < 4 ? w[l].x : w[l].y) >> (8 * (k & 3))) & 0xFFu);
                o[k] = __fmul_rn((float)q, scale);
            }
            if constexpr (sizeof(OUT) == 4) {
                float4* d = reinterpret_cast<float4*>(dst + i0);
                __stcs(d, make_float4(o[0], o[1], o[2], o[3]));
                __stcs(d + 1, make_float4(o[4], o[5], o[6], o[7]));
            } else {
                __stcs(reinterpret_cast<uint4*>(dst + i0),
                       make_uint4(tbk::pack_bf16x2(o[0], o[1]), tbk::pack_bf16x2(o[2], o[3]),
                                  tbk::pack_bf16x2(o[4], o[5]), tbk::pack_bf16x2(o[6], o[7])));
            }
        }
    }
}

// One weight per thread: elements [first, n).
template <int SRC, typename OUT>
__global__ void __launch_bounds__(kThreads)
k_dequant_one(const uint8_t* src, const float* scales, int64_t ns, int64_t gs, int64_t first,
              int64_t n, OUT* dst) {
    for (int64_t i = first + (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * kThreads) {
        int q;
        if (SRC == TB_DTYPE_INT4) {
            const uint8_t byte = src[i / 2];
            q = nibble(byte, (int)(i & 1));
        } else {
            q = (int8_t)src[i];
        }
        const float v = __fmul_rn((float)q, scale_of(scales, ns, i / gs));
        if constexpr (sizeof(OUT) == 4)
            dst[i] = v;
        else
            dst[i] = __float2bfloat16_rn(v);
    }
}

template <int SRC, typename OUT>
int launch(int64_t n, const void* src, const float* scales, int64_t ns, int64_t gs, void* dst,
           cudaStream_t s) {
    const tbh::DeviceState* ds = tbh::current_device_state();
    if (!ds) return TB_ERR_DEVICE;
    const uint8_t* q = static_cast<const uint8_t*>(src);
    OUT* out = static_cast<OUT*>(dst);
    const bool vec = (reinterpret_cast<uintptr_t>(src) % (SRC == TB_DTYPE_INT4 ? 4 : 8)) == 0 &&
                     tbh::aligned16(dst);
    int shift = -1;  // group size a power of two: a shift instead of a division
    if ((gs & (gs - 1)) == 0)
        for (shift = 0; ((int64_t)1 << shift) < gs; ++shift) {
        }
    int64_t first = 0;
    if (vec && n >= kE) {
        const int64_t nchunks = n / kE;
        // 32 CTAs per SM (several waves): measured best over 8 and 16
        k_dequant_vec<SRC, OUT><<<tbh::ew_grid((nchunks + kLoads - 1) / kLoads, kThreads, ds, 32),
                                  kThreads, 0, s>>>(q, scales, ns, gs, shift, nchunks, out);
        TB_LAUNCH_CHECK("dequant kernel");
        first = nchunks * kE;
    }
    if (first < n) {
        k_dequant_one<SRC, OUT><<<tbh::ew_grid(n - first, kThreads, ds), kThreads, 0, s>>>(
            q, scales, ns, gs, first, n, out);
        TB_LAUNCH_CHECK("dequant kernel");
    }
    return TB_OK;
}

}  // namespace

extern "C" int tb_b200_dequant(int src_dtype, int64_t n, const void* src, const float* scales,
                               int64_t n_scales, uint32_t group_size, int out_dtype, void* dst,
                               void* stream) {
    if (n < 0 || n_scales < 0) return TB_ERR_INVALID_SHAPE;
    if (n == 0) return TB_OK;
    if (!src || !dst || (n_scales > 0 && !scales)) return TB_ERR_INVALID_ARG;
    const int64_t gs = group_size > 0 ? (int64_t)group_size : n;
    cudaStream_t s = tbh::stream_of(stream);
    if (src_dtype == TB_DTYPE_INT4 && out_dtype == TB_DTYPE_F32)
        return launch<TB_DTYPE_INT4, float>(n, src, scales, n_scales, gs, dst, s);
    if (src_dtype == TB_DTYPE_INT4 && out_dtype == TB_DTYPE_BF16)
        return launch<TB_DTYPE_INT4, __nv_bfloat16>(n, src, scales, n_scales, gs, dst, s);
    if (src_dtype == TB_DTYPE_INT8 && out_dtype == TB_DTYPE_F32)
        return launch<TB_DTYPE_INT8, float>(n, src, scales, n_scales, gs, dst, s);
    if (src_dtype == TB_DTYPE_INT8 && out_dtype == TB_DTYPE_BF16)
        return launch<TB_DTYPE_INT8, __nv_bfloat16>(n, src, scales, n_scales, gs, dst, s);
    return TB_ERR_UNSUPPORTED_DTYPE;
}
