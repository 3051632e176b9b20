// k_softmax.cu -- numerically stable row softmax, with the reference's exact
// row sum.
//
// Reference arithmetic (tb_cpu_softmax_f32, src/ops/softmax.c:4-32), per row:
//   v_i   = x_i (+ mask_i)                      (one f32 add when a mask is given)
//   m     = max_i v_i  (strict '>', from -inf: NaN never becomes the max)
//   e_i   = expf(v_i - m);   sum = ((e_0 + e_1) + e_2) + ...   (f32, in order)
//   y_i   = e_i * (1.0f/sum)   if sum > 0,   else y_i = e_i
// The max is exact in any order.  The sum is reproduced bit-for-bit by the
// ordered_sum scan; expf is CUDA's full-precision expf (within 2 ulp of the C
// library's), the only source of difference from the CPU.
//
// Data path, one CTA per row: all warps take the row max (16-byte loads,
// from HBM); warp 0 recomputes e_i tile by tile and runs the ordered sum
// (re-reading the row, normally from L2); then all warps write
// y = e * (1/sum) (a third read of the row, from L2).  HBM traffic is one
// read and one write of the row.
#include <math.h>

#include "ordered_sum.cuh"
#include "tb_device.cuh"
#include "tb_internal.h"

namespace {

using tbk::Elt;

constexpr int kThreads = 256;
constexpr int kK = 8;  // terms per lane per ordered-sum tile

// Load the v_i = x_i (+ mask_i) of one VEC-wide chunk.
template <typename T, int VEC>
__device__ __forceinline__ void load_v(const T* x, const T* mask, int64_t off, float (&v)[VEC]) {
    tbk::load_vec<T, VEC>(x + off, v);
    if (mask != nullptr) {
        float mv[VEC];
        tbk::load_vec<T, VEC>(mask + off, mv);
#pragma unroll
        for (int j = 0; j < VEC; ++j) v[j] = __fadd_rn(v[j], mv[j]);
    }
}

template <typename T, int VEC>
__global__ void __launch_bounds__(kThreads)
k_softmax(const T* x, const T* mask, T* y, int64_t rows,
          int64_t cols) {
    __shared__ float red[32];
    __shared__ float row_sum;
    const int64_t row = blockIdx.x;
    const int64_t base = row * cols;
    const T* xr = x + base;
    const T* mr = mask ? mask + base : nullptr;
    T* yr = y + base;
    const int64_t nvec = cols / VEC;

    // Pass 1: row max.
    float m = -INFINITY;
    for (int64_t i = threadIdx.x; i < nvec; i += kThreads) {
        float v[VEC];
        load_v<T, VEC>(xr, mr, i * VEC, v);
#pragma unroll
        for (int j = 0; j < VEC; ++j) m = v[j] > m ? v[j] : m;
    }
    m = tbk::block_max(m, red);

    // Pass 2: warp 0, ordered sum of e_i = expf(v_i - m).
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        tbk::RunSum st;
        st.set(0.0f);
        for (int64_t t0 = 0; t0 < cols; t0 += 32 * kK) {
            float e[kK];
            const int64_t first = t0 + (int64_t)lane * kK;
            if (first + kK <= cols) {
#pragma unroll
                for (int c = 0; c < kK; c += VEC) {
                    float v[VEC];
                    load_v<T, VEC>(xr, mr, first + c, v);
#pragma unroll
                    for (int j = 0; j < VEC; ++j) e[c + j] = expf(__fsub_rn(v[j], m));
                }
            } else {
#pragma unroll
                for (int c = 0; c < kK; ++c) {
                    e[c] = 0.0f;
                    if (first + c < cols) {
                        float v[1];
                        load_v<T, 1>(xr, mr, first + c, v);
                        e[c] = expf(__fsub_rn(v[0], m));
                    }
                }
            }
            const int64_t left = cols - t0;
            tbk::ordered_sum_tile<kK>(st, e, left < 32 * kK ? (int)left : 32 * kK);
        }
        if (lane == 0) row_sum = st.s;
    }
    __syncthreads();
    const float sum = row_sum;
    const bool norm = sum > 0.0f;
    const float inv = __fdiv_rn(1.0f, sum);

    // Pass 3: y = e * inv.
    for (int64_t i = threadIdx.x; i < nvec; i += kThreads) {
        float v[VEC];
        load_v<T, VEC>(xr, mr, i * VEC, v);
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
            const float e = expf(__fsub_rn(v[j], m));
            v[j] = norm ? __fmul_rn(e, inv) : e;
        }
        tbk::store_vec<T, VEC>(yr + i * VEC, v);
    }
}

template <typename T>
int launch(int64_t rows, int64_t cols, const void* x, const void* mask, void* y, cudaStream_t s) {
    constexpr int V = Elt<T>::kVec;
    static_assert(kK % V == 0, "tile width must be a whole number of vectors");
    const T* xp = static_cast<const T*>(x);
    const T* mp = static_cast<const T*>(mask);
    T* yp = static_cast<T*>(y);
    const bool vec_ok = (cols % V == 0) && tbh::aligned16(x) && tbh::aligned16(y) &&
                        (mask == nullptr || tbh::aligned16(mask));
    if (vec_ok)
        k_softmax<T, V><<<(unsigned)rows, kThreads, 0, s>>>(xp, mp, yp, rows, cols);
    else
        k_softmax<T, 1><<<(unsigned)rows, kThreads, 0, s>>>(xp, mp, yp, rows, cols);
    TB_LAUNCH_CHECK("softmax kernel");
    return TB_OK;
}

}  // namespace

extern "C" int tb_b200_softmax(int dtype, int64_t rows, int64_t cols, const void* x,
                               const void* mask, void* y, void* stream) {
    if (rows < 0 || cols < 0 || rows > INT32_MAX) return TB_ERR_INVALID_SHAPE;
    if (rows == 0 || cols == 0) return TB_OK;
    if (!x || !y) return TB_ERR_INVALID_ARG;
    cudaStream_t s = tbh::stream_of(stream);
    if (dtype == TB_DTYPE_F32) return launch<float>(rows, cols, x, mask, y, s);
    if (dtype == TB_DTYPE_BF16) return launch<__nv_bfloat16>(rows, cols, x, mask, y, s);
    return TB_ERR_UNSUPPORTED_DTYPE;
}
