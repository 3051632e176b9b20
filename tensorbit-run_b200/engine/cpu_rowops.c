/* cpu_rowops.c -- ENGINE-SIDE code, not part of libtb_b200.so: the CPU
 * backend's slots for the five ops the b200 backend appends to TbOpType
 * (RESIDUAL_RMS_NORM, SWIGLU, ARGMAX, ROPE_ROWS, LAYER_CHAIN), written as
 * compositions of the engine's own CPU kernels (src/ops/*.c, declared in
 * include/tensorbit/run/ops.h).  With them, tb_dispatch_* of every op routes
 * for host tensors as well as device tensors.
 *
 * A maintainer adds this file to src/backend/cpu/ and calls
 * tb_cpu_rowops_fill(&cpu_backend) in tb_backend_cpu_init
 * (src/backend/cpu/registry.c:63-84) before tb_backend_register.  Host f32
 * tensors only, as the CPU kernels are f32.  Row rule of the added ops: a
 * tensor of rank >= 2 is [product of leading dims, last dim], rank 1 is one
 * row; each row goes through the kernels the reference's TransformerRunner
 * uses for one token (include/tensorbit/run/ops.hpp:79-288).
 *
 *   RESIDUAL_RMS_NORM  h = tb_cpu_residual_add_f32(x, residual), written to
 *                      h_out when given, then y = tb_cpu_rms_norm_f32(h, w)
 *   SWIGLU             out = tb_cpu_silu_f32(gate), then out[i] *= up[i]
 *                      (ops.hpp:246-248)
 *   ARGMAX             first index of the maximum, as sample_argmax
 *                      (src/main.cpp:79-89)
 *   ROPE_ROWS          tb_cpu_rope_gqa_f32 per row at positions[row]
 *   LAYER_CHAIN        the three above in one call
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "tensorbit/run/ops.h"
#include "tensorbit/run/tensor.h"
#include "tb_backend.h"

#define IN(i) (n_inputs > (i) ? (const TbTensor*)inputs[(i)] : NULL)

static int host_f32(const TbTensor* t) {
    return t == NULL || (t->device == TB_DEVICE_CPU && t->dtype == TB_DTYPE_F32 && t->data);
}

static void rows_cols(const TbTensor* t, size_t* rows, size_t* cols) {
    const size_t n = tb_tensor_nelem(t);
    *cols = t->rank >= 2 ? t->shape[t->rank - 1] : n;
    *rows = *cols ? n / *cols : 0;
}

static int residual_rms_norm_rows(TbTensor* y, TbTensor* h_out, const TbTensor* x,
                                  const TbTensor* r, const TbTensor* w, float eps) {
    size_t rows, cols;
    rows_cols(x, &rows, &cols);
    if (tb_tensor_nelem(y) != rows * cols || (r && tb_tensor_nelem(r) != rows * cols) ||
        (h_out && tb_tensor_nelem(h_out) != rows * cols) || (w && tb_tensor_nelem(w) != cols))
        return TB_ERR_INVALID_SHAPE;
    float* h = (float*)malloc(cols * sizeof(float) + 1);
    if (!h) return TB_ERR_OOM;
    int rc = TB_OK;
    for (size_t i = 0; i < rows && rc == TB_OK; i++) {
        const float* xr = tb_tensor_cf32(x) + i * cols;
        if (r)
            rc = tb_cpu_residual_add_f32(cols, xr, tb_tensor_cf32(r) + i * cols, h);
        else
            memcpy(h, xr, cols * sizeof(float));
        if (rc != TB_OK) break;
        if (h_out) memcpy(tb_tensor_f32(h_out) + i * cols, h, cols * sizeof(float));
        rc = tb_cpu_rms_norm_f32(cols, h, w ? tb_tensor_cf32(w) : NULL,
                                 tb_tensor_f32(y) + i * cols, eps);
    }
    free(h);
    return rc;
}

static int swiglu_all(TbTensor* out, const TbTensor* g, const TbTensor* u) {
    const size_t n = tb_tensor_nelem(g);
    if (tb_tensor_nelem(out) != n || tb_tensor_nelem(u) != n) return TB_ERR_INVALID_SHAPE;
    const int rc = tb_cpu_silu_f32(n, tb_tensor_cf32(g), tb_tensor_f32(out));
    if (rc != TB_OK) return rc;
    float* o = tb_tensor_f32(out);
    const float* up = tb_tensor_cf32(u);
    for (size_t i = 0; i < n; i++) o[i] *= up[i];
    return TB_OK;
}

static int rope_rows_all(TbTensor* q, TbTensor* k, const int32_t* positions, float theta,
                         int head_dim) {
    if (!positions || q->rank != 3 || k->rank != 3 || q->shape[0] != k->shape[0] ||
        q->shape[2] != k->shape[2] || (head_dim > 0 && (size_t)head_dim != q->shape[2]))
        return TB_ERR_INVALID_SHAPE;
    const size_t rows = q->shape[0], hq = q->shape[1], hkv = k->shape[1], d = q->shape[2];
    for (size_t i = 0; i < rows; i++) {
        const int rc = tb_cpu_rope_gqa_f32((int)hq, (int)hkv, (int)d, tb_tensor_f32(q) + i * hq * d,
                                           tb_tensor_f32(k) + i * hkv * d, positions[i], theta);
        if (rc != TB_OK) return rc;
    }
    return TB_OK;
}

/* RESIDUAL_RMS_NORM: output y, inputs {x, residual, weight, h_out}. */
int tb_cpu_residual_rms_norm_dispatch(void* output, const void** inputs, int n_inputs,
                                      const void* params) {
    TbTensor* y = (TbTensor*)output;
    const TbTensor* x = IN(0);
    const TbTensor* r = IN(1);
    const TbTensor* w = IN(2);
    TbTensor* h = (TbTensor*)IN(3);
    if (!y || !x || !host_f32(y) || !host_f32(x) || !host_f32(r) || !host_f32(w) || !host_f32(h))
        return TB_ERR_INVALID_ARG;
    const float eps = params ? ((const TbNormParams*)params)->eps : 1e-6f;
    return residual_rms_norm_rows(y, h, x, r, w, eps);
}

/* SWIGLU: output out, inputs {gate, up}. */
int tb_cpu_swiglu_dispatch(void* output, const void** inputs, int n_inputs, const void* params) {
    (void)params;
    TbTensor* out = (TbTensor*)output;
    const TbTensor* g = IN(0);
    const TbTensor* u = IN(1);
    if (!out || !g || !u || !host_f32(out) || !host_f32(g) || !host_f32(u))
        return TB_ERR_INVALID_ARG;
    return swiglu_all(out, g, u);
}

/* ARGMAX: output I32 [rows], inputs {logits}. */
int tb_cpu_argmax_dispatch(void* output, const void** inputs, int n_inputs, const void* params) {
    (void)params;
    TbTensor* out = (TbTensor*)output;
    const TbTensor* x = IN(0);
    if (!out || !x || !host_f32(x) || out->device != TB_DEVICE_CPU || !out->data)
        return TB_ERR_INVALID_ARG;
    if (out->dtype != TB_DTYPE_I32) return TB_ERR_UNSUPPORTED_DTYPE;
    size_t rows, cols;
    rows_cols(x, &rows, &cols);
    if (tb_tensor_nelem(out) != rows || cols == 0) return TB_ERR_INVALID_SHAPE;
    int32_t* o = (int32_t*)out->data;
    for (size_t i = 0; i < rows; i++) {
        const float* l = tb_tensor_cf32(x) + i * cols;
        size_t best = 0;
        float best_val = l[0];
        for (size_t j = 1; j < cols; j++)
            if (l[j] > best_val) {
                best_val = l[j];
                best = j;
            }
        o[i] = (int32_t)best;
    }
    return TB_OK;
}

/* ROPE_ROWS: output q [rows, n_q_heads, d], inputs {k [rows, n_kv_heads, d]}. */
int tb_cpu_rope_rows_dispatch(void* output, const void** inputs, int n_inputs,
                              const void* params) {
    TbTensor* q = (TbTensor*)output;
    TbTensor* k = (TbTensor*)IN(0);
    const TbRopeRowsParams* p = (const TbRopeRowsParams*)params;
    if (!q || !k || !p || !host_f32(q) || !host_f32(k)) return TB_ERR_INVALID_ARG;
    return rope_rows_all(q, k, p->positions, p->theta, p->head_dim);
}

/* LAYER_CHAIN: output y, inputs {h_out, act, x, residual, weight, q, k,
 * gate, up}: residual+RMSNorm, then RoPE of q/k when both are given, then
 * SwiGLU into act when gate, up and act are given. */
int tb_cpu_layer_chain_dispatch(void* output, const void** inputs, int n_inputs,
                                const void* params) {
    TbTensor* y = (TbTensor*)output;
    TbTensor* h = (TbTensor*)IN(0);
    TbTensor* act = (TbTensor*)IN(1);
    const TbTensor* x = IN(2);
    const TbTensor* r = IN(3);
    const TbTensor* w = IN(4);
    TbTensor* q = (TbTensor*)IN(5);
    TbTensor* k = (TbTensor*)IN(6);
    const TbTensor* g = IN(7);
    const TbTensor* u = IN(8);
    const TbLayerChainParams* p = (const TbLayerChainParams*)params;
    if (!p || !y || !x) return TB_ERR_INVALID_ARG;
    const TbTensor* ts[] = {y, h, act, x, r, w, q, k, g, u};
    for (int i = 0; i < 10; i++)
        if (!host_f32(ts[i])) return TB_ERR_INVALID_ARG;
    int rc = residual_rms_norm_rows(y, h, x, r, w, p->eps);
    if (rc == TB_OK && q && k) rc = rope_rows_all(q, k, p->positions, p->theta, p->head_dim);
    if (rc == TB_OK && g && u && act) rc = swiglu_all(act, g, u);
    return rc;
}

/* Fill the five added slots of the engine's CPU backend. */
void tb_cpu_rowops_fill(TbBackend* cpu) {
    cpu->ops[TB_OP_RESIDUAL_RMS_NORM] = tb_cpu_residual_rms_norm_dispatch;
    cpu->ops[TB_OP_SWIGLU] = tb_cpu_swiglu_dispatch;
    cpu->ops[TB_OP_ARGMAX] = tb_cpu_argmax_dispatch;
    cpu->ops[TB_OP_ROPE_ROWS] = tb_cpu_rope_rows_dispatch;
    cpu->ops[TB_OP_LAYER_CHAIN] = tb_cpu_layer_chain_dispatch;
}
