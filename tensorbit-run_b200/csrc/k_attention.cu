// k_attention.cu -- single-token decoder attention over a per-layer KV cache:
// the attention step of the engine's decoder forward, on the device.
//
// Reference (TransformerRunner::forward, include/tensorbit/run/ops.hpp:
// 162-204, over tb_cpu_scaled_dot_product_f32, src/ops/attention.c:5-69):
// the token's k and v go to cache row p (its position); each output row is
// one query row of a causal attention: scores s_j = (q . k_j) * scale with
// the dot product in order over the head dimension, keys past the row's own
// index masked, m = max s_j, e_j = expf(s_j - m), p_j = e_j * (1 / sum e),
// y = sum p_j v_j.  The reference runs a [cur x cur] attention (cur = p + 1)
// per head over q repeated cur times and passes the first n_heads *
// head_dim floats of the [n_heads, cur, head_dim] result on; flat row r of
// that is head r / cur at query row r % cur (TB_B200_ATTN_REFERENCE).
// TB_B200_ATTN_STANDARD computes query row p of every head (every key).
// Query head h reads k/v head h / (n_heads / n_kv_heads).
//
// One CTA per output row.  The scores give each warp a key at a time (four
// in flight), the lanes across the head dimension with a shuffle-tree sum;
// max and sum are block reductions -- orders other than the reference's
// left-to-right loops, so the results agree within f32 rounding; the weighted sum
// of v gives each warp a contiguous run of keys and each lane its own
// columns, then adds the warps' partials in warp order.  The token's own
// key and value are read from the fresh k/v vectors, and CTA 0 writes them
// into cache row p, so one launch appends and attends.  The position comes
// from device memory, so a captured CUDA graph replays unchanged.
#include <atomic>

#include "runner_kernels.h"
#include "tb_device.cuh"
#include "tb_internal.h"

namespace {

constexpr int kT = 256;
constexpr int kWarps = kT / 32;
constexpr int kMaxD = 256;  // head_dim limit: 8 columns per lane

template <int VEC>
__global__ void __launch_bounds__(kT)
k_decode_attention(int mode, int hq, int hkv, int d, int max_seq, const int32_t* __restrict__ pos_p,
                   const float* __restrict__ q, const float* __restrict__ k_new,
                   const float* __restrict__ v_new, float* kc, float* vc, float* __restrict__ out,
                   float scale, unsigned* status) {
    extern __shared__ float4 sm4[];  // 16-byte aligned for the float4 view of q
    float* sm = reinterpret_cast<float*>(sm4);
    __shared__ float red[kWarps];
    // under programmatic dependent launch, wait for the producer of q/k/v
    // (returns at once otherwise)
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int pos = *pos_p;
    if (pos < 0 || pos >= max_seq) {  // nothing is read or written
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(status, TB_B200_FLAG_POSITION_RANGE);
        return;
    }
    const int kv_dim = hkv * d, cur = pos + 1, r = blockIdx.x;
    if (r == 0) {  // the token's key and value into cache row pos
        float* kr = kc + (int64_t)pos * kv_dim;
        float* vr = vc + (int64_t)pos * kv_dim;
        for (int i = threadIdx.x; i < kv_dim; i += kT) {
            kr[i] = k_new[i];
            vr[i] = v_new[i];
        }
    }
    int h, last;
    if (mode == TB_B200_ATTN_REFERENCE) {
        h = r / cur;
        last = r % cur;
    } else {
        h = r;
        last = pos;
    }
    const int g = h / (hq / hkv);
    const int n = last + 1;  // keys 0 .. last
    float* qs = sm;               // [d]
    float* part = sm + d;         // [kWarps][d]
    float* sc = part + kWarps * d;  // [n]
    for (int i = threadIdx.x; i < d; i += kT) qs[i] = q[(int64_t)h * d + i];
    __syncthreads();

    // scores: a warp per key, lanes across the head dimension, four keys in
    // flight per warp; the lanes' partial dots meet in a shuffle tree
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float lmax = -INFINITY;
    for (int j0 = 4 * warp; j0 < n; j0 += 4 * kWarps) {
        float sj[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int j = j0 + t;
            if (j >= n) break;
            const float* kj =
                j == pos ? k_new + (int64_t)g * d : kc + (int64_t)j * kv_dim + (int64_t)g * d;
            if (VEC == 4) {
                const float4* k4 = reinterpret_cast<const float4*>(kj);
                const float4* q4 = reinterpret_cast<const float4*>(qs);
                for (int i = lane; i < d / 4; i += 32) {
                    const float4 kv = k4[i], qv = q4[i];
                    sj[t] = __fmaf_rn(qv.x, kv.x, sj[t]);
                    sj[t] = __fmaf_rn(qv.y, kv.y, sj[t]);
                    sj[t] = __fmaf_rn(qv.z, kv.z, sj[t]);
                    sj[t] = __fmaf_rn(qv.w, kv.w, sj[t]);
                }
            } else {
                for (int i = lane; i < d; i += 32) sj[t] = __fmaf_rn(qs[i], kj[i], sj[t]);
            }
        }
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int j = j0 + t;
            const float sv = __fmul_rn(tbk::warp_sum(sj[t]), scale);
            if (j < n) {
                if (lane == 0) sc[j] = sv;
                lmax = fmaxf(lmax, sv);
            }
        }
    }
    __syncthreads();  // the scores in shared memory before the other passes
    const float m = tbk::block_max(lmax, red);
    float lsum = 0.0f;
    for (int j = threadIdx.x; j < n; j += kT) {
        const float e = expf(__fsub_rn(sc[j], m));
        sc[j] = e;
        lsum = __fadd_rn(lsum, e);
    }
    const float sum = tbk::group_sum(lsum, kT, red);
    const float inv = __fdiv_rn(1.0f, sum);
    for (int j = threadIdx.x; j < n; j += kT) sc[j] = __fmul_rn(sc[j], inv);
    __syncthreads();

    // y = sum_j p_j v_j: warp w takes keys [j0, j1), lane owns columns
    // lane, lane + 32, ...
    const int per = (n + kWarps - 1) / kWarps;
    const int j0 = min(n, warp * per), j1 = min(n, j0 + per);
    float acc[kMaxD / 32];
#pragma unroll
    for (int t = 0; t < kMaxD / 32; ++t) acc[t] = 0.0f;
    for (int j = j0; j < j1; ++j) {
        const float* vj = j == pos ? v_new + (int64_t)g * d : vc + (int64_t)j * kv_dim + (int64_t)g * d;
        const float p = sc[j];
#pragma unroll
        for (int t = 0; t < kMaxD / 32; ++t) {
            const int i = lane + 32 * t;
            if (i < d) acc[t] = __fmaf_rn(p, vj[i], acc[t]);
        }
    }
#pragma unroll
    for (int t = 0; t < kMaxD / 32; ++t) {
        const int i = lane + 32 * t;
        if (i < d) part[warp * d + i] = acc[t];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < d; i += kT) {
        float y = part[i];
        for (int w = 1; w < kWarps; ++w) y = __fadd_rn(y, part[w * d + i]);
        out[(int64_t)r * d + i] = y;
    }
}

size_t smem_bytes(int d, int max_seq) {
    return ((size_t)(kWarps + 1) * d + (size_t)max_seq) * sizeof(float);
}

}  // namespace

namespace tbh {
// Opt the attention kernels in to the shared memory `max_seq` keys need
// (outside any stream capture).
int decode_attention_setup(int head_dim, int max_seq) {
    static std::atomic<size_t> granted[64];  // bytes already allowed, per device
    const size_t bytes = smem_bytes(head_dim, max_seq);
    const DeviceState* ds = current_device_state();
    if (!ds) return TB_ERR_DEVICE;
    if (bytes + kWarps * sizeof(float) > ds->smem_optin) return TB_ERR_INVALID_SHAPE;
    if (bytes <= 48 * 1024 || ds->device < 0 || ds->device >= 64 ||
        granted[ds->device].load() >= bytes)
        return TB_OK;
    TB_CUDA_TRY(cudaFuncSetAttribute(k_decode_attention<4>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    TB_CUDA_TRY(cudaFuncSetAttribute(k_decode_attention<1>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    granted[ds->device].store(bytes);
    return TB_OK;
}
}  // namespace tbh

extern "C" int tb_b200_decode_attention(int mode, int n_heads, int n_kv_heads, int head_dim,
                                        int max_seq, const int32_t* position, const float* q,
                                        const float* k, const float* v, float* k_cache,
                                        float* v_cache, float* out, void* stream) {
    return tbh::decode_attention_launch(mode, n_heads, n_kv_heads, head_dim, max_seq, position, q,
                                        k, v, k_cache, v_cache, out, tbh::stream_of(stream),
                                        false);
}

// Launch, optionally with programmatic dependent launch (the runner's step).
int tbh::decode_attention_launch(int mode, int n_heads, int n_kv_heads, int head_dim,
                                 int max_seq, const int32_t* position, const float* q,
                                 const float* k, const float* v, float* k_cache, float* v_cache,
                                 float* out, cudaStream_t s, bool pdl) {
    if (mode != TB_B200_ATTN_REFERENCE && mode != TB_B200_ATTN_STANDARD) return TB_ERR_INVALID_ARG;
    if (n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || head_dim <= 0 ||
        head_dim > kMaxD || max_seq <= 0)
        return TB_ERR_INVALID_SHAPE;
    if (!position || !q || !k || !v || !k_cache || !v_cache || !out) return TB_ERR_INVALID_ARG;
    const tbh::DeviceState* ds = tbh::current_device_state();
    if (!ds) return TB_ERR_DEVICE;
    const size_t bytes = smem_bytes(head_dim, max_seq);
    if (bytes > 48 * 1024) {
        const int rc = tbh::decode_attention_setup(head_dim, max_seq);
        if (rc != TB_OK) return rc;
    }
    const float scale = 1.f / sqrtf((float)head_dim);  // ops.hpp:175
    const bool vec = head_dim % 4 == 0 && tbh::aligned16(k) && tbh::aligned16(k_cache);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)n_heads);
    cfg.blockDim = dim3(kT);
    cfg.dynamicSmemBytes = bytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    const cudaError_t e =
        vec ? cudaLaunchKernelEx(&cfg, k_decode_attention<4>, mode, n_heads, n_kv_heads, head_dim,
                                 max_seq, position, q, k, v, k_cache, v_cache, out, scale,
                                 ds->status)
            : cudaLaunchKernelEx(&cfg, k_decode_attention<1>, mode, n_heads, n_kv_heads, head_dim,
                                 max_seq, position, q, k, v, k_cache, v_cache, out, scale,
                                 ds->status);
    tbh::count_launch();
    if (e != cudaSuccess) {
        tbh::set_error("decode attention kernel", e);
        return TB_ERR_DEVICE;
    }
    return TB_OK;
}
