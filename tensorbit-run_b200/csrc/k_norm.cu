// k_norm.cu -- residual add + RMSNorm, and RMSNorm alone, over [rows, cols].
//
// Reference: tb_cpu_residual_add_f32 (src/ops/residual.c:4-13) followed by
// tb_cpu_rms_norm_f32 (src/ops/norm.c:4-26) per row; the arithmetic and the
// register-resident data path are described at res_rms_body (bodies.cuh).
// HBM bound: 4*cols*s bytes per row (x, residual in; h, y out) plus the
// weight row once from L2.  Rows wider than the register path (more than
// 4 vectors per thread at 1024 threads) use a two-pass kernel that re-reads
// the row, normally from L2.
#include "bodies.cuh"
#include "tb_internal.h"

namespace {

using tbk::Elt;

template <typename T, int VEC, int ITEMS, int MAXT>
__global__ void __launch_bounds__(MAXT)
k_res_rms(const T* x, const T* res, const T* __restrict__ w, T* h_out, T* y, int64_t rows,
          int cols, float eps, int G) {
    __shared__ float red[32];
    tbk::res_rms_body<T, VEC, ITEMS>(x, res, w, h_out, y, rows, cols, eps, G, blockIdx.x, red);
}

// Rows wider than the register path: one CTA per row, two passes.
template <typename T>
__global__ void __launch_bounds__(1024)
k_res_rms_wide(const T* x, const T* res, const T* __restrict__ w, T* h_out, T* y, int64_t cols,
               float eps) {
    __shared__ float red[32];
    const int64_t base = (int64_t)blockIdx.x * cols;
    float ss = 0.0f;
    for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) {
        float h = Elt<T>::load(x + base + i);
        if (res) h = __fadd_rn(h, Elt<T>::load(res + base + i));
        ss = __fmaf_rn(h, h, ss);
    }
    ss = tbk::group_sum(ss, blockDim.x, red);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(__fadd_rn(ss, eps), (float)cols)));
    // Each element is re-read and then written by the same thread, so
    // in-place calls (h_out == x) stay correct.
    for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) {
        float h = Elt<T>::load(x + base + i);
        if (res) h = __fadd_rn(h, Elt<T>::load(res + base + i));
        float o = __fmul_rn(h, scale);
        if (w) o = __fmul_rn(o, Elt<T>::load(w + i));
        if (h_out) Elt<T>::store(h_out + base + i, h);
        Elt<T>::store(y + base + i, o);
    }
}

template <typename T, int VEC>
int launch_vec(const T* x, const T* res, const T* w, T* h, T* y, int64_t rows, int64_t cols,
               float eps, cudaStream_t s) {
    const tbh::NormCfg c = tbh::norm_cfg(cols / VEC, 1024);
    const int rows_per_cta = c.threads / c.G;
    const unsigned grid = (unsigned)((rows + rows_per_cta - 1) / rows_per_cta);
    const int n = (int)cols;
    if (c.items == 0) {
        k_res_rms_wide<T><<<(unsigned)rows, 1024, 0, s>>>(x, res, w, h, y, cols, eps);
    } else if (c.threads <= 256) {
        switch (c.items) {
            case 1: k_res_rms<T, VEC, 1, 256><<<grid, c.threads, 0, s>>>(x, res, w, h, y, rows, n, eps, c.G); break;
            case 2: k_res_rms<T, VEC, 2, 256><<<grid, c.threads, 0, s>>>(x, res, w, h, y, rows, n, eps, c.G); break;
            default: k_res_rms<T, VEC, 4, 256><<<grid, c.threads, 0, s>>>(x, res, w, h, y, rows, n, eps, c.G); break;
        }
    } else {
        switch (c.items) {
            case 1: k_res_rms<T, VEC, 1, 1024><<<grid, c.threads, 0, s>>>(x, res, w, h, y, rows, n, eps, c.G); break;
            case 2: k_res_rms<T, VEC, 2, 1024><<<grid, c.threads, 0, s>>>(x, res, w, h, y, rows, n, eps, c.G); break;
            default: k_res_rms<T, VEC, 4, 1024><<<grid, c.threads, 0, s>>>(x, res, w, h, y, rows, n, eps, c.G); break;
        }
    }
    TB_LAUNCH_CHECK("residual_rms_norm kernel");
    return TB_OK;
}

template <typename T>
int launch(const void* x, const void* res, const void* w, void* h, void* y, int64_t rows,
           int64_t cols, float eps, cudaStream_t s) {
    constexpr int V = Elt<T>::kVec;
    const bool vec_ok = (cols % V == 0) && tbh::aligned16(x) && (!res || tbh::aligned16(res)) &&
                        (!w || tbh::aligned16(w)) && (!h || tbh::aligned16(h)) &&
                        tbh::aligned16(y);
    const T* xp = static_cast<const T*>(x);
    const T* rp = static_cast<const T*>(res);
    const T* wp = static_cast<const T*>(w);
    T* hp = static_cast<T*>(h);
    T* yp = static_cast<T*>(y);
    if (vec_ok) return launch_vec<T, V>(xp, rp, wp, hp, yp, rows, cols, eps, s);
    return launch_vec<T, 1>(xp, rp, wp, hp, yp, rows, cols, eps, s);
}

int run(int dtype, int64_t rows, int64_t cols, const void* x, const void* res, const void* w,
        void* h, void* y, float eps, void* stream) {
    if (rows < 0 || cols < 0 || rows > INT32_MAX || cols > INT32_MAX) return TB_ERR_INVALID_SHAPE;
    if (rows == 0 || cols == 0) return TB_OK;
    if (!x || !y) return TB_ERR_INVALID_ARG;
    cudaStream_t s = tbh::stream_of(stream);
    if (dtype == TB_DTYPE_F32) return launch<float>(x, res, w, h, y, rows, cols, eps, s);
    if (dtype == TB_DTYPE_BF16) return launch<__nv_bfloat16>(x, res, w, h, y, rows, cols, eps, s);
    return TB_ERR_UNSUPPORTED_DTYPE;
}

}  // namespace

extern "C" int tb_b200_residual_rms_norm(int dtype, int64_t rows, int64_t cols, const void* x,
                                         const void* residual, const void* weight, void* h_out,
                                         void* y, float eps, void* stream) {
    return run(dtype, rows, cols, x, residual, weight, h_out, y, eps, stream);
}

extern "C" int tb_b200_rms_norm(int dtype, int64_t rows, int64_t cols, const void* x,
                                const void* weight, void* y, float eps, void* stream) {
    return run(dtype, rows, cols, x, nullptr, weight, nullptr, y, eps, stream);
}
