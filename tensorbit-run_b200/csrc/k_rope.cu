// k_rope.cu -- interleaved-pair rotary embedding of Q and K rows, in place.
//
// Reference (tb_cpu_rope_gqa_f32, src/ops/rope.c:43-81), per token at
// `position`, per head, per pair i < head_dim/2:
//   f_i = 1.0f / powf(theta, (2.0f*i)/(float)head_dim)
//   c = cosf((float)position * f_i),  s = sinf((float)position * f_i)
//   (a0, a1) = (v[2i], v[2i+1])  ->  (a0*c - a1*s, a1*c + a0*s)
// cos/sin come from a table built on the host with the same C library calls
// in the same expressions (tb_b200_rope_table), so inside the table the
// result is bit-identical to the reference.  Outside it, f_i is still host
// computed, the angle is the same f32 product, and cos/sin are CUDA's
// full-precision sincosf (within 2 ulp of the C library).
//
// Data path: one CTA per token row (see rope_body, bodies.cuh).  HBM bound:
// 2*(Hq+Hkv)*d*s bytes per row, plus 4*d bytes of L2-resident table.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "bodies.cuh"
#include "tb_internal.h"

namespace {

using tbk::Elt;
using tbk::RopeConst;

template <typename T, int VEC, int MODE, int UNROLL>
__global__ void __launch_bounds__(256)
k_rope(T* q, T* k, const int32_t* __restrict__ positions, int hq, int hkv, int d,
       const float2* __restrict__ table, int table_pos, const __grid_constant__ RopeConst rc) {
    tbk::rope_body<T, VEC, MODE, UNROLL>(q, k, positions, hq, hkv, d, table, table_pos, rc,
                                         blockIdx.x);
}

template <typename T, int MODE>
int launch(int64_t rows, int hq, int hkv, int d, void* q, void* k, const int32_t* positions,
           const float* table, int table_pos, const RopeConst& rc, cudaStream_t s) {
    constexpr int V = Elt<T>::kVec;
    T* qp = static_cast<T*>(q);
    T* kp = static_cast<T*>(k);
    const float2* tp = reinterpret_cast<const float2*>(table);
    const bool vec_ok = (d % V == 0) && (!hq || tbh::aligned16(q)) && (!hkv || tbh::aligned16(k)) &&
                        (table == nullptr || tbh::aligned16(table));
    // d <= 512: at most 256 lanes per head, so 256 threads always cover a head.
    const int threads = 256;
    if (vec_ok)
        k_rope<T, V, MODE, 4><<<(unsigned)rows, threads, 0, s>>>(qp, kp, positions, hq, hkv, d, tp,
                                                                 table_pos, rc);
    else
        k_rope<T, 2, MODE, 4><<<(unsigned)rows, threads, 0, s>>>(qp, kp, positions, hq, hkv, d, tp,
                                                                 table_pos, rc);
    TB_LAUNCH_CHECK("rope kernel");
    return TB_OK;
}

int check_shape(int64_t rows, int hq, int hkv, int d) {
    if (rows < 0 || hq < 0 || hkv < 0 || d < 0) return TB_ERR_INVALID_SHAPE;
    if (d / 2 > tbk::kRopeMaxPairs || rows > INT32_MAX) return TB_ERR_INVALID_SHAPE;
    return TB_OK;
}

}  // namespace

namespace tbh {
// f_i exactly as src/ops/rope.c:52 computes it, with the host C library.
void rope_inv_freq(float theta, int head_dim, float* out) {
    for (int i = 0; i < head_dim / 2; i++)
        out[i] = 1.0f / powf(theta, (2.0f * i) / (float)head_dim);
}
}  // namespace tbh

extern "C" int tb_b200_rope_table(float theta, int head_dim, int n_positions, float* table_dev,
                                  void* stream) {
    if (head_dim < 2 || n_positions < 0 || head_dim / 2 > tbk::kRopeMaxPairs)
        return TB_ERR_INVALID_SHAPE;
    if (n_positions == 0) return TB_OK;
    if (!table_dev) return TB_ERR_INVALID_ARG;
    const int half = head_dim / 2;
    const size_t n = (size_t)n_positions * half * 2;
    float* host = (float*)malloc(n * sizeof(float));
    if (!host) return TB_ERR_OOM;
    float freq[tbk::kRopeMaxPairs];
    tbh::rope_inv_freq(theta, head_dim, freq);
    for (int p = 0; p < n_positions; p++) {
        float* row = host + (size_t)p * half * 2;
        for (int i = 0; i < half; i++) {
            row[2 * i] = cosf((float)p * freq[i]);
            row[2 * i + 1] = sinf((float)p * freq[i]);
        }
    }
    cudaStream_t s = tbh::stream_of(stream);
    cudaError_t e = cudaMemcpyAsync(table_dev, host, n * sizeof(float), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    free(host);
    if (e != cudaSuccess) {
        tbh::set_error("rope table upload", e);
        return TB_ERR_DEVICE;
    }
    return TB_OK;
}

extern "C" int tb_b200_rope_rows(int dtype, int64_t rows, int n_q_heads, int n_kv_heads,
                                 int head_dim, void* q, void* k, const int32_t* positions,
                                 float theta, const float* table, int table_positions,
                                 void* stream) {
    int rc = check_shape(rows, n_q_heads, n_kv_heads, head_dim);
    if (rc) return rc;
    if (dtype != TB_DTYPE_F32 && dtype != TB_DTYPE_BF16) return TB_ERR_UNSUPPORTED_DTYPE;
    if (rows == 0 || head_dim < 2 || n_q_heads + n_kv_heads == 0) return TB_OK;
    if ((n_q_heads && !q) || (n_kv_heads && !k) || !positions) return TB_ERR_INVALID_ARG;
    RopeConst c;
    memset(&c, 0, sizeof c);
    tbh::rope_inv_freq(theta, head_dim, c.inv_freq);
    cudaStream_t s = tbh::stream_of(stream);
    if (dtype == TB_DTYPE_F32)
        return launch<float, tbk::kRopePerRow>(rows, n_q_heads, n_kv_heads, head_dim, q, k,
                                               positions, table, table_positions, c, s);
    return launch<__nv_bfloat16, tbk::kRopePerRow>(rows, n_q_heads, n_kv_heads, head_dim, q, k,
                                                   positions, table, table_positions, c, s);
}

extern "C" int tb_b200_rope(int dtype, int n_q_heads, int n_kv_heads, int head_dim, void* q,
                            void* k, int position, float theta, void* stream) {
    int rc = check_shape(1, n_q_heads, n_kv_heads, head_dim);
    if (rc) return rc;
    if (dtype != TB_DTYPE_F32 && dtype != TB_DTYPE_BF16) return TB_ERR_UNSUPPORTED_DTYPE;
    if (head_dim < 2 || n_q_heads + n_kv_heads == 0) return TB_OK;
    if ((n_q_heads && !q) || (n_kv_heads && !k)) return TB_ERR_INVALID_ARG;
    RopeConst c;
    memset(&c, 0, sizeof c);
    tbh::rope_inv_freq(theta, head_dim, c.inv_freq);
    for (int i = 0; i < head_dim / 2; i++) {
        c.cs[i].x = cosf((float)position * c.inv_freq[i]);
        c.cs[i].y = sinf((float)position * c.inv_freq[i]);
    }
    cudaStream_t s = tbh::stream_of(stream);
    if (dtype == TB_DTYPE_F32)
        return launch<float, tbk::kRopeConst>(1, n_q_heads, n_kv_heads, head_dim, q, k, nullptr,
                                              nullptr, 0, c, s);
    return launch<__nv_bfloat16, tbk::kRopeConst>(1, n_q_heads, n_kv_heads, head_dim, q, k, nullptr,
                                                  nullptr, 0, c, s);
}
