// k_linear.cu -- y = W x (+ bias) for one f32 input vector, dense or with an
// N:M mask: the engine's linear layers (GEMV), on the device.
//
// Reference (src/ops/linear.c:4-53): y[j] = bias[j] (or 0) + sum of
// x[i] * w[j][i], accumulated left to right in f32.  Sparse: in / M groups
// per row, one mask byte per group, bit k (k < M) keeps weight g*M + k; a
// bit past 7 never matches the byte, and columns past (in / M) * M are not
// used.  The weights are stored dense (pruned ones 0), so both forms read
// all of W.
//
// One warp per output: the lanes stream the row as 16-byte loads (four in
// flight), the input vector comes through L1, each lane accumulates with
// FMAs and a shuffle tree adds the lanes -- a different summation order
// from the reference's, so results agree within the f32 row tolerance (the
// same magnitude of rounding as the reference's own chain), not bit for bit.
// HBM bound: out * in * 4 bytes of W per call.
#include "tb_device.cuh"
#include "tb_internal.h"

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kU = 4;  // 16-byte loads of W in flight per lane

// Weight idx of a row is kept: its group is a whole group and its bit set.
__device__ __forceinline__ bool kept(const uint8_t* mr, int64_t idx, int m, int64_t used) {
    if (idx >= used) return false;
    const int k = (int)(idx % m);
    return (mr[idx / m] & (uint8_t)(1u << k)) != 0;
}

template <bool SPARSE, bool VEC>
__global__ void __launch_bounds__(kThreads)
k_linear(int64_t out_f, int64_t in_f, const float* __restrict__ x, const float* __restrict__ w,
         const uint8_t* __restrict__ mask, const float* __restrict__ bias, float* __restrict__ y,
         int m) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * kWarps;
    const int64_t groups = SPARSE ? in_f / m : 0;
    const int64_t used = SPARSE ? groups * m : in_f;
    for (int64_t j = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); j < out_f; j += warps) {
        const float* wr = w + j * in_f;
        const uint8_t* mr = SPARSE ? mask + j * groups : nullptr;
        float acc = 0.0f;
        if (VEC) {
            const int64_t nv = used / 4;  // whole float4s of used weights
            const float4* w4 = reinterpret_cast<const float4*>(wr);
            const float4* x4 = reinterpret_cast<const float4*>(x);
            for (int64_t v0 = lane; v0 < nv; v0 += 32 * kU) {
                float4 wv[kU];
                uint32_t mb4[kU];  // the 2:4 case: each float4's mask byte, loaded beside it
#pragma unroll
                for (int u = 0; u < kU; ++u) {
                    const int64_t v = v0 + 32 * u;
                    wv[u] = v < nv ? __ldcs(w4 + v) : make_float4(0.f, 0.f, 0.f, 0.f);
                    mb4[u] = SPARSE && m == 4 && v < nv ? __ldcs(mr + v) : 0u;
                }
#pragma unroll
                for (int u = 0; u < kU; ++u) {
                    const int64_t v = v0 + 32 * u;
                    if (v >= nv) break;
                    const float4 xv = __ldg(x4 + v);
                    if (SPARSE) {
                        const int64_t i = 4 * v;
                        if (m == 4) {  // the common 2:4 case: one mask byte per float4
                            const uint32_t mb = mb4[u];
                            if (mb & 1u) acc = __fmaf_rn(xv.x, wv[u].x, acc);
                            if (mb & 2u) acc = __fmaf_rn(xv.y, wv[u].y, acc);
                            if (mb & 4u) acc = __fmaf_rn(xv.z, wv[u].z, acc);
                            if (mb & 8u) acc = __fmaf_rn(xv.w, wv[u].w, acc);
                        } else {
                            if (kept(mr, i, m, used)) acc = __fmaf_rn(xv.x, wv[u].x, acc);
                            if (kept(mr, i + 1, m, used)) acc = __fmaf_rn(xv.y, wv[u].y, acc);
                            if (kept(mr, i + 2, m, used)) acc = __fmaf_rn(xv.z, wv[u].z, acc);
                            if (kept(mr, i + 3, m, used)) acc = __fmaf_rn(xv.w, wv[u].w, acc);
                        }
                    } else {
                        acc = __fmaf_rn(xv.x, wv[u].x, acc);
                        acc = __fmaf_rn(xv.y, wv[u].y, acc);
                        acc = __fmaf_rn(xv.z, wv[u].z, acc);
                        acc = __fmaf_rn(xv.w, wv[u].w, acc);
                    }
                }
            }
            for (int64_t i = nv * 4 + lane; i < used; i += 32)  // used not a multiple of 4
                if (!SPARSE || kept(mr, i, m, used)) acc = __fmaf_rn(x[i], wr[i], acc);
        } else {
            for (int64_t i = lane; i < used; i += 32)
                if (!SPARSE || kept(mr, i, m, used)) acc = __fmaf_rn(x[i], wr[i], acc);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(tbk::kFull, acc, o));
        if (lane == 0) y[j] = bias ? __fadd_rn(bias[j], acc) : acc;
    }
}

template <bool SPARSE>
int launch(int64_t out_f, int64_t in_f, const float* x, const float* w, const uint8_t* mask,
           const float* bias, float* y, int m, cudaStream_t s) {
    const tbh::DeviceState* ds = tbh::current_device_state();
    if (!ds) return TB_ERR_DEVICE;
    const int grid = tbh::ew_grid(out_f, kWarps, ds, 16);  // one warp per output row
    const bool vec = in_f % 4 == 0 && tbh::aligned16(x) && tbh::aligned16(w);
    if (vec)
        k_linear<SPARSE, true><<<grid, kThreads, 0, s>>>(out_f, in_f, x, w, mask, bias, y, m);
    else
        k_linear<SPARSE, false><<<grid, kThreads, 0, s>>>(out_f, in_f, x, w, mask, bias, y, m);
    TB_LAUNCH_CHECK("linear kernel");
    return TB_OK;
}

}  // namespace

extern "C" int tb_b200_sparse_linear(int64_t out_features, int64_t in_features, const float* x,
                                     const float* w, const uint8_t* mask, const float* bias,
                                     float* y, int nm_n, int nm_m, void* stream) {
    if (!x || !w || !mask || !y) return TB_ERR_INVALID_ARG;   // linear.c:10
    if (nm_m < 2 || nm_n >= nm_m) return TB_ERR_INVALID_ARG;  // linear.c:11
    if (out_features < 0 || in_features < 0) return TB_ERR_INVALID_SHAPE;
    if (out_features == 0) return TB_OK;
    return launch<true>(out_features, in_features, x, w, mask, bias, y, nm_m,
                        tbh::stream_of(stream));
}

extern "C" int tb_b200_dense_linear(int64_t out_features, int64_t in_features, const float* x,
                                    const float* w, const float* bias, float* y, void* stream) {
    if (!x || !w || !y) return TB_ERR_INVALID_ARG;  // linear.c:41
    if (out_features < 0 || in_features < 0) return TB_ERR_INVALID_SHAPE;
    if (out_features == 0) return TB_OK;
    return launch<false>(out_features, in_features, x, w, nullptr, bias, y, 4,
                         tbh::stream_of(stream));
}
