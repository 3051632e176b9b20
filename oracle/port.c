/*
 * port.c -- CPU restatement of the reference's per-vector row kernels.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h).  Each function restates one
 * reference kernel with the same arithmetic in the same evaluation order, so
 * that, compiled with the reference's flags (-O3 -mavx2 -mfma -std=gnu11,
 * which let gcc contract a*b+c into an FMA exactly as it does for the
 * reference), it returns bit-identical results.  tests/test_oracle.py checks
 * that against the reference's own objects (oracle/_ref) and against the
 * committed golden checksums.
 *
 * Error codes are the reference's TbError values
 * (include/tensorbit/run/common.h:54-71): 0 = TB_OK, 8 = TB_ERR_INVALID_ARG.
 */
#include "oracle.h"

#include <math.h>
#include <string.h>

#define ORC_OK 0
#define ORC_ERR_INVALID_ARG 8

/* sqrt(2/pi) as the reference spells it (include/tensorbit/run/common.h:218). */
#define ORC_SQRT_2_PI 0.79788456080286535588f

/*
 * RMSNorm, src/ops/norm.c:4-26.
 * The accumulator is seeded with eps (norm.c:8), squares are accumulated
 * left to right (norm.c:9-11), the scale is 1/sqrtf(acc/n) (norm.c:13) and
 * each output is (x*scale)*weight, evaluated left to right (norm.c:17).
 */
int orc_rms_norm_f32(size_t n, const float* x, const float* weight, float* y, float eps) {
    if (x == NULL || y == NULL) return ORC_ERR_INVALID_ARG;
    float acc = eps;
    for (size_t i = 0; i < n; i++) acc += x[i] * x[i];
    const float scale = 1.0f / sqrtf(acc / (float)n);
    if (weight != NULL) {
        for (size_t i = 0; i < n; i++) y[i] = x[i] * scale * weight[i];
    } else {
        for (size_t i = 0; i < n; i++) y[i] = x[i] * scale;
    }
    return ORC_OK;
}

/* Residual add, src/ops/residual.c:4-13: y = x + residual. */
int orc_residual_add_f32(size_t n, const float* x, const float* residual, float* y) {
    if (x == NULL || residual == NULL || y == NULL) return ORC_ERR_INVALID_ARG;
    for (size_t i = 0; i < n; i++) y[i] = x[i] + residual[i];
    return ORC_OK;
}

/*
 * tanh-GELU, src/ops/activation.c:4-16:
 *   v3 = v*v*v; inner = sqrt(2/pi)*(v + 0.044715*v3); y = 0.5*v*(1 + tanhf(inner)).
 */
int orc_gelu_f32(size_t n, const float* x, float* y) {
    if (x == NULL || y == NULL) return ORC_ERR_INVALID_ARG;
    for (size_t i = 0; i < n; i++) {
        const float v = x[i];
        const float cube = v * v * v;
        const float arg = ORC_SQRT_2_PI * (v + 0.044715f * cube);
        const float t = tanhf(arg);
        y[i] = 0.5f * v * (1.0f + t);
    }
    return ORC_OK;
}

/* SiLU, src/ops/activation.c:18-27: y = v / (1 + expf(-v)), a true division. */
int orc_silu_f32(size_t n, const float* x, float* y) {
    if (x == NULL || y == NULL) return ORC_ERR_INVALID_ARG;
    for (size_t i = 0; i < n; i++) {
        const float v = x[i];
        y[i] = v / (1.0f + expf(-v));
    }
    return ORC_OK;
}

/*
 * SwiGLU as the engine composes it: silu(gate, gate) at
 * include/tensorbit/run/ops.hpp:246, then gate[i] *= up[i] at ops.hpp:247-248.
 */
int orc_swiglu_f32(size_t n, const float* gate, const float* up, float* out) {
    if (gate == NULL || up == NULL || out == NULL) return ORC_ERR_INVALID_ARG;
    int rc = orc_silu_f32(n, gate, out);
    if (rc != ORC_OK) return rc;
    for (size_t i = 0; i < n; i++) out[i] *= up[i];
    return ORC_OK;
}

/*
 * One head of the interleaved-pair rotation of src/ops/rope.c:51-61 (Q) and
 * rope.c:67-77 (K): for pair i, (a0, a1) = (v[2i], v[2i+1]) becomes
 * (a0*c - a1*s, a1*c + a0*s).  gcc makes no FMA out of these expressions in
 * the reference's own loop (each product is rounded, then added), so
 * contraction is switched off here to keep the same rounding when this
 * loop is vectorised.
 */
__attribute__((noinline, optimize("fp-contract=off")))
static void orc_rotate_head(float* v, int half, const float* c, const float* s) {
    for (int i = 0; i < half; i++) {
        const float a0 = v[2 * i];
        const float a1 = v[2 * i + 1];
        v[2 * i] = a0 * c[i] - a1 * s[i];
        v[2 * i + 1] = a1 * c[i] + a0 * s[i];
    }
}

/*
 * GQA RoPE for one token, src/ops/rope.c:43-81.
 * Frequency i is 1.0f/powf(base, (2.0f*i)/(float)head_dim) (rope.c:52,68) and
 * the angle is (float)position * frequency (rope.c:53-54,69-70).  The
 * reference recomputes powf/cosf/sinf for every head; the values do not
 * depend on the head, so they are computed once per pair here (identical
 * bits, one libm call per pair instead of one per pair and head).
 * Q has n_q_heads rows of head_dim, K has n_kv_heads rows of head_dim.
 */
int orc_rope_gqa_f32(int n_q_heads, int n_kv_heads, int head_dim, float* q, float* k,
                     int position, float theta_base) {
    if (q == NULL || k == NULL) return ORC_ERR_INVALID_ARG;
    const int half = head_dim / 2;
    float cbuf[1024], sbuf[1024];
    if (half > 1024) return ORC_ERR_INVALID_ARG;
    for (int i = 0; i < half; i++) {
        const float freq = 1.0f / powf(theta_base, (2.0f * i) / (float)head_dim);
        cbuf[i] = cosf((float)position * freq);
        sbuf[i] = sinf((float)position * freq);
    }
    for (int h = 0; h < n_q_heads; h++) orc_rotate_head(q + (size_t)h * head_dim, half, cbuf, sbuf);
    for (int h = 0; h < n_kv_heads; h++) orc_rotate_head(k + (size_t)h * head_dim, half, cbuf, sbuf);
    return ORC_OK;
}

/*
 * Numerically stable softmax, src/ops/softmax.c:4-32.
 * Pass 1 takes the maximum of x (+ mask) with a strict '>' starting from
 * -INFINITY (softmax.c:8-13).  Pass 2 stores e = expf(v - max) and adds it to
 * an fp32 running sum strictly left to right (softmax.c:15-22).  Pass 3
 * multiplies by 1.0f/sum, and only when sum > 0 (softmax.c:24-29), so a NaN
 * or zero sum leaves the unnormalised exponentials in y.
 */
int orc_softmax_f32(size_t n, const float* x, const float* mask, float* y) {
    if (x == NULL || y == NULL) return ORC_ERR_INVALID_ARG;
    float top = -INFINITY;
    for (size_t i = 0; i < n; i++) {
        float v = x[i];
        if (mask != NULL) v += mask[i];
        if (v > top) top = v;
    }
    float total = 0.0f;
    for (size_t i = 0; i < n; i++) {
        float v = x[i];
        if (mask != NULL) v += mask[i];
        const float e = expf(v - top);
        y[i] = e;
        total += e;
    }
    if (total > 0.0f) {
        const float inv = 1.0f / total;
        for (size_t i = 0; i < n; i++) y[i] *= inv;
    }
    return ORC_OK;
}

/*
 * Embedding gather, src/ops/embedding.c:4-14: row t of y is a byte copy of
 * row token_ids[t] of the table.  The reference does no range check; callers
 * of this oracle pass in-range ids only.
 */
int orc_embedding_f32(const int* token_ids, int n_tokens, int embedding_dim, const float* table,
                      float* y) {
    if (token_ids == NULL || table == NULL || y == NULL) return ORC_ERR_INVALID_ARG;
    for (int t = 0; t < n_tokens; t++) {
        const int id = token_ids[t];
        memcpy(y + (size_t)t * embedding_dim, table + (size_t)id * embedding_dim,
               sizeof(float) * (size_t)embedding_dim);
    }
    return ORC_OK;
}

/*
 * Greedy argmax, src/main.cpp:79-89 (static there): start from element 0 and
 * move only on a strictly greater value, so the first maximum wins and a NaN
 * never wins (a NaN at index 0 keeps index 0).
 */
int orc_argmax_f32(const float* logits, int n) {
    int best = 0;
    float best_v = logits[0];
    for (int i = 1; i < n; i++) {
        if (logits[i] > best_v) {
            best_v = logits[i];
            best = i;
        }
    }
    return best;
}

/*
 * bf16 conversion used for the bf16-I/O variants: widen is exact; narrowing
 * rounds to nearest, ties to even, on the top 16 bits of the IEEE-754 single.
 */
float orc_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

uint16_t orc_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, sizeof u);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u);
    const uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}

/*
 * N:M-masked and dense f32 linear (GEMV), src/ops/linear.c:4-53:
 *   y[j] = bias[j] (or 0) + sum over kept i of x[i] * w[j][i], accumulated
 *   left to right in f32 (gcc contracts each step into an FMA with the
 *   reference's flags).  Sparse: in / M groups per row, one mask byte per
 *   group, bit k (k < M) keeps weight g*M + k (linear.c:16-27); a bit past 7
 *   never matches the byte, and columns past (in / M) * M are not used.
 */
int orc_sparse_linear_f32(size_t out_features, size_t in_features, const float* x, const float* w,
                          const uint8_t* mask, const float* bias, float* y, int nm_n, int nm_m) {
    if (!x || !w || !mask || !y) return ORC_ERR_INVALID_ARG;
    if (nm_m < 2 || nm_n >= nm_m) return ORC_ERR_INVALID_ARG;
    const size_t groups = in_features / (size_t)nm_m;
    for (size_t j = 0; j < out_features; j++) {
        float acc = bias ? bias[j] : 0.0f;
        const float* wr = w + j * in_features;
        const uint8_t* mr = mask + j * groups;
        for (size_t g = 0; g < groups; g++) {
            const uint8_t mb = mr[g];
            for (int k = 0; k < nm_m; k++)
                if (mb & (uint8_t)(1u << k)) acc += x[g * nm_m + k] * wr[g * nm_m + k];
        }
        y[j] = acc;
    }
    return ORC_OK;
}

int orc_dense_linear_f32(size_t out_features, size_t in_features, const float* x, const float* w,
                         const float* bias, float* y) {
    if (!x || !w || !y) return ORC_ERR_INVALID_ARG;
    for (size_t j = 0; j < out_features; j++) {
        float acc = bias ? bias[j] : 0.0f;
        const float* wr = w + j * in_features;
        for (size_t i = 0; i < in_features; i++) acc += x[i] * wr[i];
        y[j] = acc;
    }
    return ORC_OK;
}
