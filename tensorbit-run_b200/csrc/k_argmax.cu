// k_argmax.cu -- greedy argmax of each row, bit-exact with the reference.
//
// Reference semantics (sample_argmax, src/main.cpp:79-89): start at index 0
// and move only on a strictly greater value.  Equivalently:
//   - if x_0 is NaN nothing compares greater than it: the answer is 0;
//   - otherwise the answer is the smallest index whose value equals the
//     maximum of the non-NaN values (+0 and -0 compare equal, so the first
//     zero wins), and 0 when no value exceeds -inf.
// Each thread scans its elements in increasing index order with a strict
// '>' (so it keeps its first maximum), and partial results combine by
// (larger value, else smaller index) -- an order-independent rule with the
// same answer as the sequential scan.
//
// Data path: HBM bound, R*V*s bytes read once.  Rows with many columns get
// one CTA each; short rows share a CTA one warp per row.
#include <math.h>

#include "tb_device.cuh"
#include "tb_internal.h"

namespace {

using tbk::Elt;
constexpr int kNone = 0x7fffffff;

struct Best {
    float v;
    int i;
};

__device__ __forceinline__ void take(Best& b, float v, int i) {
    if (v > b.v) {
        b.v = v;
        b.i = i;
    }
}

__device__ __forceinline__ Best better(Best a, Best b) {
    if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
    return a;
}

__device__ __forceinline__ Best warp_best(Best b) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        Best other;
        other.v = __shfl_xor_sync(tbk::kFull, b.v, o);
        other.i = __shfl_xor_sync(tbk::kFull, b.i, o);
        b = better(b, other);
    }
    return b;
}

// Scan elements [lo, hi) of a row with stride `step` vectors.
template <typename T, int VEC>
__device__ __forceinline__ Best scan(const T* xr, int64_t nvec, int64_t first, int step) {
    Best b{-INFINITY, kNone};
    for (int64_t i = first; i < nvec; i += step) {
        float v[VEC];
        tbk::load_vec_stream<T, VEC>(xr + i * VEC, v);
#pragma unroll
        for (int j = 0; j < VEC; ++j) take(b, v[j], (int)(i * VEC + j));
    }
    return b;
}

__device__ __forceinline__ int finish(Best b, float x0) {
    if (x0 != x0) return 0;  // NaN at index 0 is never beaten
    return b.i == kNone ? 0 : b.i;
}

// One CTA per row.
template <typename T, int VEC>
__global__ void __launch_bounds__(512)
k_argmax_cta(const T* __restrict__ x, int32_t* __restrict__ out, int64_t cols) {
    __shared__ float sv[32];
    __shared__ int si[32];
    const T* xr = x + (int64_t)blockIdx.x * cols;
    Best b = scan<T, VEC>(xr, cols / VEC, threadIdx.x, blockDim.x);
    b = warp_best(b);
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        sv[warp] = b.v;
        si[warp] = b.i;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        Best r{sv[0], si[0]};
        for (int w = 1; w < nw; ++w) r = better(r, Best{sv[w], si[w]});
        out[blockIdx.x] = finish(r, Elt<T>::load(xr));
    }
}

// One warp per row.
template <typename T, int VEC>
__global__ void __launch_bounds__(256)
k_argmax_warp(const T* __restrict__ x, int32_t* __restrict__ out, int64_t rows, int64_t cols) {
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const T* xr = x + row * cols;
    Best b = warp_best(scan<T, VEC>(xr, cols / VEC, threadIdx.x & 31, 32));
    if ((threadIdx.x & 31) == 0) out[row] = finish(b, Elt<T>::load(xr));
}

template <typename T>
int launch(int64_t rows, int64_t cols, const void* x, int32_t* out, cudaStream_t s) {
    constexpr int V = Elt<T>::kVec;
    const T* xp = static_cast<const T*>(x);
    const bool vec_ok = (cols % V == 0) && tbh::aligned16(x);
    const bool narrow = cols <= 2048;
    if (narrow) {
        const unsigned grid = (unsigned)((rows + 7) / 8);
        if (vec_ok)
            k_argmax_warp<T, V><<<grid, 256, 0, s>>>(xp, out, rows, cols);
        else
            k_argmax_warp<T, 1><<<grid, 256, 0, s>>>(xp, out, rows, cols);
    } else {
        if (vec_ok)
            k_argmax_cta<T, V><<<(unsigned)rows, 512, 0, s>>>(xp, out, cols);
        else
            k_argmax_cta<T, 1><<<(unsigned)rows, 512, 0, s>>>(xp, out, cols);
    }
    TB_LAUNCH_CHECK("argmax kernel");
    return TB_OK;
}

}  // namespace

extern "C" int tb_b200_argmax(int dtype, int64_t rows, int64_t cols, const void* x, int32_t* out,
                              void* stream) {
    if (rows < 0 || cols < 0 || rows > INT32_MAX || cols > INT32_MAX) return TB_ERR_INVALID_SHAPE;
    if (rows == 0) return TB_OK;
    if (cols == 0) return TB_ERR_INVALID_SHAPE;  // the reference reads logits[0]
    if (!x || !out) return TB_ERR_INVALID_ARG;
    cudaStream_t s = tbh::stream_of(stream);
    if (dtype == TB_DTYPE_F32) return launch<float>(rows, cols, x, out, s);
    if (dtype == TB_DTYPE_BF16) return launch<__nv_bfloat16>(rows, cols, x, out, s);
    return TB_ERR_UNSUPPORTED_DTYPE;
}
