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
#include "tma.cuh"

namespace {

constexpr int kT = 256;
constexpr int kWarps = kT / 32;
constexpr int kMaxD = 256;  // head_dim limit: 8 columns per lane
constexpr int kPrefetchRows = 1024;  // cache rows asked of L2 ahead of the wait
constexpr int kKeys = 8;             // keys in flight per warp
constexpr int kSlots = kMaxD / 128;  // float4 columns per lane
constexpr int kSplitMin = 512;       // rows of more keys are split over CTAs
constexpr int kMaxSplits = 16;

template <int VEC>
__global__ void __launch_bounds__(kT)
k_decode_attention(int mode, int hq, int hkv, int d, int max_seq, const int32_t* __restrict__ pos_p,
                   const float* __restrict__ q, const float* __restrict__ k_new,
                   const float* __restrict__ v_new, float* kc, float* vc, float* __restrict__ out,
                   float scale, unsigned* status, float* part_g, int* count_g) {
    extern __shared__ float4 sm4[];  // 16-byte aligned for the float4 view of q
    float* sm = reinterpret_cast<float*>(sm4);
    __shared__ float red[kWarps];
    if (VEC == 4) {
        // The earlier tokens' cache rows do not depend on the kernel this
        // launch may overlap (programmatic dependent launch): ask L2 for this
        // row's keys and values first.  The position is read early too: it
        // only changes at the end of a decoder step.
        const int p0 = *pos_p;
        if (p0 > 0 && p0 < max_seq) {
            const int cur0 = p0 + 1, r0 = blockIdx.x;
            const int h0 = mode == TB_B200_ATTN_REFERENCE ? r0 / cur0 : r0;
            const int last0 = mode == TB_B200_ATTN_REFERENCE ? r0 % cur0 : p0;
            const int64_t off = (int64_t)(h0 / (hq / hkv)) * d;
            const int n0 = last0 + 1, ns = gridDim.y;
            int a0 = 0, a1 = n0;
            if (ns > 1 && n0 > kSplitMin) {
                a0 = (int)((int64_t)blockIdx.y * n0 / ns);
                a1 = (int)((int64_t)(blockIdx.y + 1) * n0 / ns);
            } else if (blockIdx.y != 0) {
                a1 = 0;
            }
            a1 = min(min(a1, p0), a0 + kPrefetchRows);  // row p0 is the new one
            for (int j = a0 + (int)threadIdx.x; j < a1; j += kT) {
                tbk::prefetch_l2(kc + (int64_t)j * hkv * d + off, (uint32_t)d * 4);
                tbk::prefetch_l2(vc + (int64_t)j * hkv * d + off, (uint32_t)d * 4);
            }
        }
    }
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
    if (r == 0 && blockIdx.y == 0) {  // the token's key and value into cache row pos
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
    // A long row is split over the gridDim.y CTAs of its row: each takes
    // keys [k0, k1) and leaves (max, sum, unnormalised weighted v) in part_g;
    // the last to finish combines them.  Rows of at most kSplitMin keys are
    // done whole by the first CTA (the others leave at once).
    const int ns = gridDim.y, sp = blockIdx.y;
    const bool split = ns > 1 && n > kSplitMin;
    if (!split && sp != 0) return;
    const int k0 = split ? (int)((int64_t)sp * n / ns) : 0;
    const int k1 = split ? (int)((int64_t)(sp + 1) * n / ns) : n;
    const int nk = k1 - k0;
    float* qs = sm;               // [d]
    float* part = sm + d;         // [kWarps][d]
    float* sc = part + kWarps * d;  // [nk]: scores of keys k0 .. k1-1
    for (int i = threadIdx.x; i < d; i += kT) qs[i] = q[(int64_t)h * d + i];
    __syncthreads();

    // scores: a warp per key, lanes across the head dimension (float4
    // columns lane and lane + 32), eight keys in flight per warp; the lanes'
    // partial dots meet in a shuffle tree
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int d4 = d / 4;
    float lmax = -INFINITY;
    for (int j0 = k0 + kKeys * warp; j0 < k1; j0 += kKeys * kWarps) {
        float sj[kKeys];
        if (VEC == 4) {
            const float4* q4 = reinterpret_cast<const float4*>(qs);
            float4 kv[kKeys][kSlots];
#pragma unroll
            for (int t = 0; t < kKeys; ++t) {
                const int j = j0 + t;
                const float4* k4 = reinterpret_cast<const float4*>(
                    j == pos ? k_new + (int64_t)g * d : kc + (int64_t)j * kv_dim + (int64_t)g * d);
#pragma unroll
                for (int u = 0; u < kSlots; ++u) {
                    const int i = lane + 32 * u;
                    kv[t][u] = j < k1 && i < d4 ? k4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
#pragma unroll
            for (int t = 0; t < kKeys; ++t) {
                sj[t] = 0.0f;
#pragma unroll
                for (int u = 0; u < kSlots; ++u) {
                    const int i = lane + 32 * u;
                    if (i >= d4) break;
                    const float4 qv = q4[i];
                    sj[t] = __fmaf_rn(qv.x, kv[t][u].x, sj[t]);
                    sj[t] = __fmaf_rn(qv.y, kv[t][u].y, sj[t]);
                    sj[t] = __fmaf_rn(qv.z, kv[t][u].z, sj[t]);
                    sj[t] = __fmaf_rn(qv.w, kv[t][u].w, sj[t]);
                }
            }
        } else {
#pragma unroll
            for (int t = 0; t < kKeys; ++t) {
                sj[t] = 0.0f;
                const int j = j0 + t;
                if (j >= k1) continue;
                const float* kj =
                    j == pos ? k_new + (int64_t)g * d : kc + (int64_t)j * kv_dim + (int64_t)g * d;
                for (int i = lane; i < d; i += 32) sj[t] = __fmaf_rn(qs[i], kj[i], sj[t]);
            }
        }
#pragma unroll
        for (int t = 0; t < kKeys; ++t) {
            const int j = j0 + t;
            const float sv = __fmul_rn(tbk::warp_sum(sj[t]), scale);
            if (j < k1) {
                if (lane == 0) sc[j - k0] = sv;
                lmax = fmaxf(lmax, sv);
            }
        }
    }
    __syncthreads();  // the scores in shared memory before the other passes
    const float m = tbk::block_max(lmax, red);
    float lsum = 0.0f;
    for (int j = threadIdx.x; j < nk; j += kT) {
        const float e = expf(__fsub_rn(sc[j], m));
        sc[j] = e;
        lsum = __fadd_rn(lsum, e);
    }
    const float sum = tbk::group_sum(lsum, kT, red);
    if (!split) {  // whole row: p = e * (1 / sum), as the reference
        const float inv = __fdiv_rn(1.0f, sum);
        for (int j = threadIdx.x; j < nk; j += kT) sc[j] = __fmul_rn(sc[j], inv);
    }
    __syncthreads();

    // y = sum_j p_j v_j: warp w takes keys [j0, j1) in order, eight in
    // flight; a lane owns float4 columns lane and lane + 32 (scalar columns
    // lane, lane + 32, ... when the rows are not float4-aligned)
    const int per = (nk + kWarps - 1) / kWarps;
    const int j0 = k0 + min(nk, warp * per), j1 = k0 + min(nk, warp * per + per);
    if (VEC == 4) {
        float4 acc[kSlots];
#pragma unroll
        for (int u = 0; u < kSlots; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j = j0; j < j1; j += kKeys) {
            float4 vv[kKeys][kSlots];
            float pj[kKeys];
#pragma unroll
            for (int t = 0; t < kKeys; ++t) {
                const int jj = j + t;
                pj[t] = jj < j1 ? sc[jj - k0] : 0.0f;
                const float4* v4 = reinterpret_cast<const float4*>(
                    jj == pos ? v_new + (int64_t)g * d : vc + (int64_t)jj * kv_dim + (int64_t)g * d);
#pragma unroll
                for (int u = 0; u < kSlots; ++u) {
                    const int i = lane + 32 * u;
                    vv[t][u] = jj < j1 && i < d4 ? v4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
#pragma unroll
            for (int t = 0; t < kKeys; ++t) {
                if (j + t >= j1) break;
#pragma unroll
                for (int u = 0; u < kSlots; ++u) {
                    acc[u].x = __fmaf_rn(pj[t], vv[t][u].x, acc[u].x);
                    acc[u].y = __fmaf_rn(pj[t], vv[t][u].y, acc[u].y);
                    acc[u].z = __fmaf_rn(pj[t], vv[t][u].z, acc[u].z);
                    acc[u].w = __fmaf_rn(pj[t], vv[t][u].w, acc[u].w);
                }
            }
        }
        float4* part4 = reinterpret_cast<float4*>(part + warp * d);
#pragma unroll
        for (int u = 0; u < kSlots; ++u) {
            const int i = lane + 32 * u;
            if (i < d4) part4[i] = acc[u];
        }
    } else {
        float acc[kMaxD / 32];
#pragma unroll
        for (int t = 0; t < kMaxD / 32; ++t) acc[t] = 0.0f;
        for (int j = j0; j < j1; ++j) {
            const float* vj =
                j == pos ? v_new + (int64_t)g * d : vc + (int64_t)j * kv_dim + (int64_t)g * d;
            const float p = sc[j - k0];
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
    }
    __syncthreads();
    if (!split) {
        for (int i = threadIdx.x; i < d; i += kT) {
            float y = part[i];
            for (int w = 1; w < kWarps; ++w) y = __fadd_rn(y, part[w * d + i]);
            out[(int64_t)r * d + i] = y;
        }
        return;
    }
    // this CTA's partial: max, sum, weighted v (d floats)
    float* mine = part_g + ((int64_t)r * ns + sp) * (d + 2);
    for (int i = threadIdx.x; i < d; i += kT) {
        float y = part[i];
        for (int w = 1; w < kWarps; ++w) y = __fadd_rn(y, part[w * d + i]);
        mine[2 + i] = y;
    }
    if (threadIdx.x == 0) {
        mine[0] = m;
        mine[1] = sum;
    }
    __threadfence();
    __syncthreads();
    __shared__ int last_cta;
    if (threadIdx.x == 0) last_cta = atomicAdd(count_g + r, 1) == ns - 1;
    __syncthreads();
    if (!last_cta) return;
    // the last CTA of the row combines the parts in split order
    __threadfence();
    const float* row_parts = part_g + (int64_t)r * ns * (d + 2);
    float mg = -INFINITY;
    for (int k = 0; k < ns; ++k) mg = fmaxf(mg, __ldcg(row_parts + (int64_t)k * (d + 2)));
    float tot = 0.0f;
    for (int k = 0; k < ns; ++k) {
        const float* pk = row_parts + (int64_t)k * (d + 2);
        tot = __fadd_rn(tot, __fmul_rn(__ldcg(pk + 1), expf(__fsub_rn(__ldcg(pk), mg))));
    }
    const float inv = __fdiv_rn(1.0f, tot);
    for (int i = threadIdx.x; i < d; i += kT) {
        float y = 0.0f;
        for (int k = 0; k < ns; ++k) {
            const float* pk = row_parts + (int64_t)k * (d + 2);
            y = __fmaf_rn(__ldcg(pk + 2 + i), expf(__fsub_rn(__ldcg(pk), mg)), y);
        }
        out[(int64_t)r * d + i] = __fmul_rn(y, inv);
    }
    if (threadIdx.x == 0) count_g[r] = 0;  // ready for the next launch
}

size_t smem_bytes(int d, int max_seq) {
    return ((size_t)(kWarps + 1) * d + (size_t)max_seq) * sizeof(float);
}

}  // namespace

namespace tbh {
// CTAs per row for long rows: about two per SM over the rows, at most
// kMaxSplits, none when no row can exceed kSplitMin keys.
int decode_attention_splits(int n_rows, int max_seq) {
    const DeviceState* ds = current_device_state();
    if (!ds || max_seq <= kSplitMin || n_rows <= 0) return 1;
    int sp = 2 * ds->sm_count / n_rows;
    return sp < 1 ? 1 : sp > kMaxSplits ? kMaxSplits : sp;
}

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
                                        false, 1, nullptr, nullptr);
}

// Launch, optionally with programmatic dependent launch (the runner's step).
int tbh::decode_attention_launch(int mode, int n_heads, int n_kv_heads, int head_dim,
                                 int max_seq, const int32_t* position, const float* q,
                                 const float* k, const float* v, float* k_cache, float* v_cache,
                                 float* out, cudaStream_t s, bool pdl, int splits, float* part,
                                 int* counters) {
    if (splits < 1 || splits > kMaxSplits || (splits > 1 && (!part || !counters)))
        return TB_ERR_INVALID_ARG;
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
    // The float4 path reads k, v and both caches as float4 (the new token's
    // k and v too): every one of them must start on a 16-byte boundary --
    // slices of a packed qkv buffer may not.
    const bool vec = head_dim % 4 == 0 && tbh::aligned16(k) && tbh::aligned16(k_cache) &&
                     tbh::aligned16(v) && tbh::aligned16(v_cache);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)n_heads, (unsigned)splits);
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
                                 ds->status, part, counters)
            : cudaLaunchKernelEx(&cfg, k_decode_attention<1>, mode, n_heads, n_kv_heads, head_dim,
                                 max_seq, position, q, k, v, k_cache, v_cache, out, scale,
                                 ds->status, part, counters);
    tbh::count_launch();
    if (e != cudaSuccess) {
        tbh::set_error("decode attention kernel", e);
        return TB_ERR_DEVICE;
    }
    return TB_OK;
}
