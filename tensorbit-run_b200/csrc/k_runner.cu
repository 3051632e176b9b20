// k_runner.cu -- the fused kernels of the device decoder step (runner.cu):
// one GEMV launch per group of projections that share an input, with the
// step that follows each group folded into its epilogue, and the RMSNorm of
// the state vector.
//
// Reference steps (TransformerRunner::forward, include/tensorbit/run/
// ops.hpp) and the epilogue that replaces each:
//   q, k, v = W x; rope(q, k) at the position         (:140-159)  kRope
//   x = x + Wo attn                                    (:207-218)  kResidual
//   g = silu(Wg x_mlp) * (Wu x_mlp)                    (:226-248)  kSwiglu
//   x = x + Wd g                                       (:250-256)  kResidual
//   logits = Wlm x; position += 1                      (:269-284)  kPlain
// The arithmetic of each epilogue is the separate kernel's: the rotation of
// tbk::rope_rotate over the host-built cos/sin table, tbk::silu_f(g) * u, and
// one f32 add for the residual.
//
// Each warp computes two output rows (gemv.cuh): two consecutive rows of a
// projection -- for q and k exactly the pair (2i, 2i+1) RoPE rotates
// together -- or row j of the gate and up projections.  Every kernel here is
// launched with programmatic dependent launch: a CTA first asks L2 to fetch
// its first rows of weights (they do not depend on the previous kernel),
// then waits (griddepcontrol.wait) for the previous kernel's results, so the
// weight stream starts during that kernel's tail.
#include "bodies.cuh"
#include "gemv.cuh"
#include "tb_internal.h"
#include "tma.cuh"

#include <utility>

#include "runner_kernels.h"

namespace {

using tbh::GemvArgs;

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

__device__ __forceinline__ void pdl_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Unit u -> (segment, first row, second row).  A unit is two consecutive
// rows of one segment (the last row twice when a segment's count is odd),
// or for kSwiglu row u of segment 0 (gate) and of segment 1 (up).
template <int EPI>
__device__ __forceinline__ bool unit_rows(const GemvArgs& a, int64_t u, int& s, int64_t& r0,
                                          int64_t& r1) {
    if constexpr (EPI == tbh::kSwiglu) {
        if (u >= a.seg[0].rows) return false;
        s = 0;
        r0 = r1 = u;
        return true;
    } else {
        for (s = 0; s < a.nseg; ++s) {
            const int64_t n = (a.seg[s].rows + 1) / 2;
            if (u < n) {
                r0 = 2 * u;
                r1 = r0 + 1 < a.seg[s].rows ? r0 + 1 : r0;
                return true;
            }
            u -= n;
        }
        return false;
    }
}

// Weight words per row of a quantized layout.
template <int LAYOUT>
__host__ __device__ constexpr int64_t qwords(int64_t cols) {
    return LAYOUT == tbh::kInt8 ? cols / 4 : cols / 8;
}

template <int LAYOUT>
__device__ __forceinline__ void row_ptrs(const tbh::GemvSeg& g, int64_t cols, int64_t r,
                                         const float4*& v, const uint8_t*& ib) {
    if (LAYOUT == tbh::kDense) {
        v = static_cast<const float4*>(g.w) + r * (cols / 4);
        ib = nullptr;
    } else if (LAYOUT == tbh::kInt8 || LAYOUT == tbh::kInt4) {  // v: the row's first word
        v = reinterpret_cast<const float4*>(static_cast<const uint32_t*>(g.w) +
                                            r * qwords<LAYOUT>(cols));
        ib = nullptr;
    } else {
        const int64_t pairs = cols / 8;
        v = static_cast<const float4*>(g.w) + r * pairs;
        ib = g.idx + r * tbk::packed_idx_stride(pairs);
    }
}

// L2 prefetch of the start of one weight row: enough for the warp's first
// step, little enough that the prefetches of every resident warp stay far
// below the L2 (whole rows of a 200 MB projection group would evict each
// other).  Sizes are multiples of 16 bytes; rows start 16-byte aligned.
template <int LAYOUT>
__device__ __forceinline__ void prefetch_row(int64_t cols, const float4* v, const uint8_t* ib,
                                             int64_t step) {
    constexpr int64_t kCap = 2048;
    if (LAYOUT == tbh::kInt8 || LAYOUT == tbh::kInt4) {
        const int64_t woff = step * tbk::kQStep;
        const int64_t left = (qwords<LAYOUT>(cols) - woff) * 4;
        if (left > 0)
            tbk::prefetch_l2(reinterpret_cast<const uint32_t*>(v) + woff, (uint32_t)min(left, kCap));
        return;
    }
    const int64_t off = step * tbk::kGemvStep;  // float4s (dense) or pairs (packed)
    if (LAYOUT == tbh::kDense) {
        const int64_t left = (cols / 4 - off) * 16;
        if (left > 0) tbk::prefetch_l2(v + off, (uint32_t)min(left, kCap));
    } else {
        const int64_t pairs = cols / 8;
        const int64_t left = (pairs - off) * 16;
        if (left > 0) {
            tbk::prefetch_l2(v + off, (uint32_t)min(left, kCap));
            tbk::prefetch_l2(ib + off, (uint32_t)min(tbk::packed_idx_stride(pairs) - off, kCap));
        }
    }
}

// Four CTAs per SM (64 registers a thread): measured faster than the
// uncapped build (64-128 registers) and than caps of 3, 5 or 6.
template <int LAYOUT, int EPI, bool NORM>
__global__ void __launch_bounds__(kThreads, 4) k_fgemv(const __grid_constant__ GemvArgs a) {
    extern __shared__ float4 xs[];  // NORM: the normalised x
    __shared__ float red[kWarps];
    __shared__ float2 psum[kWarps];  // split rows: each warp's partial sums
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    // a.ks warps share a unit, each over a contiguous range of its steps
    const int ks = a.ks, upc = kWarps / ks, slot = wid / ks, part = wid % ks;
    const int64_t per_row = (LAYOUT == tbh::kInt8 || LAYOUT == tbh::kInt4)
                                ? qwords<LAYOUT>(a.cols) / tbk::kQStep + 1
                                : (LAYOUT == tbh::kDense ? a.cols / 4 : a.cols / 8) / tbk::kGemvStep + 1;
    const int64_t s0 = part * per_row / ks, s1 = (part + 1) * per_row / ks;
    {  // weights do not depend on the previous kernel: start their stream
        int s;
        int64_t r0, r1;
        if (lane == 0 && unit_rows<EPI>(a, (int64_t)blockIdx.x * upc + slot, s, r0, r1)) {
            const float4* v;
            const uint8_t* ib;
            const tbh::GemvSeg& g0 = a.seg[s];
            row_ptrs<LAYOUT>(g0, a.cols, r0, v, ib);
            prefetch_row<LAYOUT>(a.cols, v, ib, s0);
            const tbh::GemvSeg& g1 = EPI == tbh::kSwiglu ? a.seg[1] : a.seg[s];
            row_ptrs<LAYOUT>(g1, a.cols, r1, v, ib);
            prefetch_row<LAYOUT>(a.cols, v, ib, s0);
        }
    }
    pdl_wait();
    if (a.advance && blockIdx.x == 0 && threadIdx.x == 0) *a.advance += 1;
    const float4* x4 = reinterpret_cast<const float4*>(a.x);
    const int64_t n4 = a.cols / 4;
    if constexpr (NORM) {
        // rms_norm(x) * w (src/ops/norm.c:4-26): every CTA sums the squares
        // in the same order, so all hold the same scale
        float ss = 0.0f;
        for (int64_t i = threadIdx.x; i < n4; i += kThreads) {
            const float4 v = x4[i];
            ss = __fmaf_rn(v.x, v.x, ss);
            ss = __fmaf_rn(v.y, v.y, ss);
            ss = __fmaf_rn(v.z, v.z, ss);
            ss = __fmaf_rn(v.w, v.w, ss);
        }
        ss = tbk::group_sum(ss, kThreads, red);
        const float scale =
            __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(__fadd_rn(ss, a.eps), (float)a.cols)));
        const float4* w4 = reinterpret_cast<const float4*>(a.norm_w);
        float4* out4 = blockIdx.x == 0 ? reinterpret_cast<float4*>(a.norm_out) : nullptr;
        for (int64_t i = threadIdx.x; i < n4; i += kThreads) {
            float4 v = x4[i];
            v.x = __fmul_rn(v.x, scale);
            v.y = __fmul_rn(v.y, scale);
            v.z = __fmul_rn(v.z, scale);
            v.w = __fmul_rn(v.w, scale);
            if (w4) {
                const float4 w = w4[i];
                v.x = __fmul_rn(v.x, w.x);
                v.y = __fmul_rn(v.y, w.y);
                v.z = __fmul_rn(v.z, w.z);
                v.w = __fmul_rn(v.w, w.w);
            }
            xs[i] = v;
            if (out4) out4[i] = v;
        }
        __syncthreads();
    }
    int pos = 0;
    if (EPI == tbh::kRope) pos = *a.pos;
    const float4* xsrc = NORM ? xs : x4;
    // the loop bound is the same for every warp of the CTA (it synchronises)
    for (int64_t base = (int64_t)blockIdx.x * upc; base < a.units; base += (int64_t)gridDim.x * upc) {
        int s = 0;
        int64_t r0 = 0, r1 = 0;
        const bool have = unit_rows<EPI>(a, base + slot, s, r0, r1);
        float a0 = 0.0f, a1 = 0.0f;
        if (have) {
            const tbh::GemvSeg& g0 = a.seg[s];
            const tbh::GemvSeg& g1 = EPI == tbh::kSwiglu ? a.seg[1] : a.seg[s];
            const float4 *v0, *v1;
            const uint8_t *i0, *i1;
            row_ptrs<LAYOUT>(g0, a.cols, r0, v0, i0);
            row_ptrs<LAYOUT>(g1, a.cols, r1, v1, i1);
            if (LAYOUT == tbh::kDense)
                tbk::dense_dot2<NORM>(v0, v1, n4, xsrc, lane, a0, a1, s0, s1);
            else if (LAYOUT == tbh::kPacked)
                tbk::packed_dot2<NORM>(v0, i0, v1, i1, a.cols / 8, xsrc, lane, a0, a1, s0, s1);
            else
                tbk::quant_dot2<LAYOUT == tbh::kInt8 ? 8 : 4, NORM>(
                    reinterpret_cast<const uint32_t*>(v0), reinterpret_cast<const uint32_t*>(v1),
                    tbk::QRow{g0.scales, g0.gshift, (uint32_t)(r0 * a.cols)},
                    tbk::QRow{g1.scales, g1.gshift, (uint32_t)(r1 * a.cols)},
                    qwords<LAYOUT>(a.cols), xsrc, lane, a0, a1, s0, s1);
        }
        tbk::warp_sum2(a0, a1);
        if (ks > 1) {  // the unit's parts, added in part order
            if (lane == 0) psum[wid] = make_float2(a0, a1);
            __syncthreads();
            if (part == 0) {
                a0 = psum[wid].x;
                a1 = psum[wid].y;
                for (int k = 1; k < ks; ++k) {
                    a0 = __fadd_rn(a0, psum[wid + k].x);
                    a1 = __fadd_rn(a1, psum[wid + k].y);
                }
            }
            __syncthreads();
        }
        if (!have || part != 0 || lane != 0) continue;
        const tbh::GemvSeg& g0 = a.seg[s];
        if (EPI == tbh::kSwiglu) {
            a.act[r0] = __fmul_rn(tbk::silu_f(a0), a1);
        } else if (EPI == tbh::kResidual) {
            g0.y[r0] = __fadd_rn(a.res[r0], a0);
            if (r1 != r0) g0.y[r1] = __fadd_rn(a.res[r1], a1);
        } else {
            if (EPI == tbh::kRope && s < a.rope_segs && r1 != r0) {
                if (pos >= 0 && pos < a.rope_positions) {
                    const int half = a.head_dim / 2;
                    const float2 cs = a.rope[(int64_t)pos * half + (r0 % a.head_dim) / 2];
                    tbk::rope_rotate(a0, a1, cs.x, cs.y);
                } else {
                    atomicOr(a.status, TB_B200_FLAG_POSITION_RANGE);
                }
            }
            g0.y[r0] = a0;
            if (r1 != r0) g0.y[r1] = a1;
        }
    }
}

// RMSNorm of one vector (tb_cpu_rms_norm_f32, src/ops/norm.c:4-26): one CTA.
__global__ void __launch_bounds__(1024)
k_rnorm(int64_t n, const float* x, const float* __restrict__ w, float* y, float eps) {
    __shared__ float red[32];
    pdl_wait();
    float ss = 0.0f;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) ss = __fmaf_rn(x[i], x[i], ss);
    ss = tbk::group_sum(ss, blockDim.x, red);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(__fadd_rn(ss, eps), (float)n)));
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        float o = __fmul_rn(x[i], scale);
        if (w) o = __fmul_rn(o, w[i]);
        y[i] = o;
    }
}

template <typename... P, typename... A>
int launch_pdl(void (*kernel)(P...), int grid, int threads, size_t smem, cudaStream_t s,
               A&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3((unsigned)threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<A>(args)...);
    tbh::count_launch();
    if (e != cudaSuccess) {
        tbh::set_error("runner kernel launch", e);
        return TB_ERR_DEVICE;
    }
    return TB_OK;
}

template <int LAYOUT, int EPI>
int fgemv_norm(const GemvArgs& a, int grid, cudaStream_t s) {
    if (a.norm)
        return launch_pdl(k_fgemv<LAYOUT, EPI, true>, grid, kThreads, (size_t)a.cols * 4, s, a);
    return launch_pdl(k_fgemv<LAYOUT, EPI, false>, grid, kThreads, 0, s, a);
}

template <int LAYOUT>
int fgemv_layout(const GemvArgs& a, int epi, int grid, cudaStream_t s) {
    switch (epi) {
        case tbh::kPlain: return fgemv_norm<LAYOUT, tbh::kPlain>(a, grid, s);
        case tbh::kResidual: return fgemv_norm<LAYOUT, tbh::kResidual>(a, grid, s);
        case tbh::kRope: return fgemv_norm<LAYOUT, tbh::kRope>(a, grid, s);
        case tbh::kSwiglu: return fgemv_norm<LAYOUT, tbh::kSwiglu>(a, grid, s);
        default: return TB_ERR_INVALID_ARG;
    }
}

template <int LAYOUT, int EPI>
cudaError_t allow_smem(int bytes) {
    return cudaFuncSetAttribute(k_fgemv<LAYOUT, EPI, true>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

}  // namespace

namespace tbh {

int fused_gemv(const GemvArgs& a, int layout, int epi, cudaStream_t s) {
    const DeviceState* ds = current_device_state();
    if (!ds) return TB_ERR_DEVICE;
    if (a.nseg < 1 || a.nseg > 3 || (epi == kSwiglu && a.nseg != 2)) return TB_ERR_INVALID_ARG;
    GemvArgs b = a;
    int64_t units = 0;
    if (epi == kSwiglu) {
        if (a.seg[0].rows != a.seg[1].rows) return TB_ERR_INVALID_SHAPE;
        units = a.seg[0].rows;
    } else {
        for (int i = 0; i < a.nseg; ++i) units += (a.seg[i].rows + 1) / 2;
    }
    if (units == 0) return TB_OK;
    // split rows over more warps when there are few of them (two resident
    // CTAs of 8 warps per SM), at most one part per step of a row
    const int64_t steps =
        layout == kInt8   ? qwords<kInt8>(a.cols) / tbk::kQStep + 1
        : layout == kInt4 ? qwords<kInt4>(a.cols) / tbk::kQStep + 1
                          : (layout == kDense ? a.cols / 4 : a.cols / 8) / tbk::kGemvStep + 1;
    int ks = 1;
    while (ks < kWarps && units * ks < (int64_t)ds->sm_count * 2 * kWarps && 2 * ks <= steps) ks *= 2;
    b.units = units;
    b.ks = ks;
    const int upc = kWarps / ks;
    // one wave of resident CTAs (four per SM): each normalises x once and
    // loops over units (measured faster than two waves of 8 per SM)
    const int grid = ew_grid(units, upc, ds, 4);
    switch (layout) {
        case kDense: return fgemv_layout<kDense>(b, epi, grid, s);
        case kPacked: return fgemv_layout<kPacked>(b, epi, grid, s);
        case kInt8: return fgemv_layout<kInt8>(b, epi, grid, s);
        case kInt4: return fgemv_layout<kInt4>(b, epi, grid, s);
        default: return TB_ERR_INVALID_ARG;
    }
}

int runner_norm(int64_t n, const float* x, const float* w, float* y, float eps, cudaStream_t s) {
    return launch_pdl(k_rnorm, 1, 1024, 0, s, n, x, w, y, eps);
}

// The normalising variants keep x (cols floats) in shared memory.
int fused_gemv_setup(int64_t cols) {
    const DeviceState* ds = current_device_state();
    if (!ds) return TB_ERR_DEVICE;
    const size_t bytes = (size_t)cols * 4;
    if (bytes + 64 > ds->smem_optin) return TB_ERR_INVALID_SHAPE;
    if (bytes <= 48 * 1024) return TB_OK;
    const int b = (int)bytes;
    cudaError_t e = cudaSuccess;
    const cudaError_t r[] = {allow_smem<kDense, kPlain>(b),   allow_smem<kDense, kResidual>(b),
                             allow_smem<kDense, kRope>(b),    allow_smem<kDense, kSwiglu>(b),
                             allow_smem<kPacked, kPlain>(b),  allow_smem<kPacked, kResidual>(b),
                             allow_smem<kPacked, kRope>(b),   allow_smem<kPacked, kSwiglu>(b),
                             allow_smem<kInt8, kPlain>(b),    allow_smem<kInt8, kResidual>(b),
                             allow_smem<kInt8, kRope>(b),     allow_smem<kInt8, kSwiglu>(b),
                             allow_smem<kInt4, kPlain>(b),    allow_smem<kInt4, kResidual>(b),
                             allow_smem<kInt4, kRope>(b),     allow_smem<kInt4, kSwiglu>(b)};
    for (cudaError_t x : r)
        if (x != cudaSuccess) e = x;
    if (e != cudaSuccess) {
        set_error("fused GEMV shared memory", e);
        return TB_ERR_DEVICE;
    }
    return TB_OK;
}

}  // namespace tbh
