/*
 * runner.c -- CPU restatement of the engine's single-token decoder forward,
 * tensorbit::run::TransformerRunner::forward
 * (include/tensorbit/run/ops.hpp:79-288).
 *
 * TEST INFRASTRUCTURE ONLY: the answer the device runner is checked against,
 * and the CPU baseline of the decoder benchmark.  It is pinned to the
 * reference's own TransformerRunner (compiled from the reference tree by
 * oracle/Makefile into oracle/_ref/libpinrunner.so) by tests/test_oracle.py.
 *
 * Per token (ops.hpp line numbers):
 *   x = embed[token]                                            :92
 *   per layer whose q/k/v weights exist (:109):
 *     x = rms_norm(x) * input_norm                              :119
 *     q, k, v = W x   (sparse 2:4 when the layer has a mask)    :140-149
 *     rope(q, k) at the current position                        :159
 *     k, v -> cache row pos                                     :162-169
 *     attention -> attn_out                                     :172-204
 *     x = x + Wo attn_out                                       :207-218
 *     x_mlp = rms_norm(x) * post_norm                           :221-223
 *     g = silu(Wg x_mlp) * (Wu x_mlp); x = x + Wd g             :226-256
 *   x = rms_norm(x) * final_norm; logits = Wlm x                :260-281
 *
 * Attention rows.  For position p (cur = p + 1 keys) the reference runs a
 * causal [cur x cur] attention per head over q repeated cur times and hands
 * the FIRST n_heads * head_dim floats of that [n_heads, cur, head_dim]
 * result to the output projection (:185-218).  Flat row r < n_heads of it is
 * head r / cur at query row r % cur, which attends keys 0 .. r % cur.
 * ORC_ATTN_REFERENCE computes exactly those rows; ORC_ATTN_STANDARD computes
 * row p of every head (the usual decoder attention).  Each row follows
 * src/ops/attention.c:5-69: scores by an in-order dot product times scale,
 * keys past the row set to -inf, max, expf, an in-order sum, 1/sum, and an
 * in-order weighted sum of v over all keys.
 *
 * Where the reference reads outside its buffers this restatement takes the
 * defined choice the device runner takes, and the parity tests avoid those
 * inputs:
 *   - rms_norm runs over the state vector, max(hidden, vocab) floats
 *     (:39, src/backend/cpu/norm.c:12), with weights of hidden floats: here
 *     the norm covers hidden floats (identical when vocab <= hidden);
 *   - at position 0 head h reads k/v head h (:176), past k and v for
 *     h >= n_kv_heads: here head h reads k/v head h / (n_heads / n_kv_heads)
 *     (identical when n_kv_heads == n_heads);
 *   - a layer without a mask reads mask bytes from whatever follows its
 *     weights (Model::get_mask never returns an empty tensor, model.hpp:163):
 *     here such a layer is dense.  Masked layers always run as 2:4 groups
 *     (the dispatcher passes no N:M parameters, src/backend/cpu/registry.c:93).
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "oracle.h"

#define ORC_OK 0
#define ORC_ERR_INVALID_ARG 8
#define ORC_ERR_OOM 7

/* y = W x for one projection: sparse 2:4 over its mask, or dense. */
static int orc_project(const orc_lin* w, const float* x, float* y) {
    if (w->mask)
        return orc_sparse_linear_f32((size_t)w->rows, (size_t)w->cols, x, w->w, w->mask, NULL, y,
                                     2, 4);
    return orc_dense_linear_f32((size_t)w->rows, (size_t)w->cols, x, w->w, NULL, y);
}

/* One query row of src/ops/attention.c:5-69: keys 0 .. seq_len-1 at
 * kbase + j * stride (v likewise), keys past `last` masked to -inf. */
static int orc_attention_row(const float* q, const float* kbase, const float* vbase, size_t stride,
                             int seq_len, int last, int head_dim, float scale, float* scores,
                             float* y) {
    for (int j = 0; j < seq_len; j++) {
        const float* kj = kbase + (size_t)j * stride;
        float s = 0.0f;
        for (int d = 0; d < head_dim; d++) s += q[d] * kj[d];
        s *= scale;
        if (j > last) s = -INFINITY;
        scores[j] = s;
    }
    float max_val = -INFINITY;
    for (int j = 0; j < seq_len; j++)
        if (scores[j] > max_val) max_val = scores[j];
    float sum = 0.0f;
    for (int j = 0; j < seq_len; j++) {
        const float e = expf(scores[j] - max_val);
        scores[j] = e;
        sum += e;
    }
    const float inv_sum = 1.0f / sum;
    for (int j = 0; j < seq_len; j++) scores[j] *= inv_sum;
    for (int d = 0; d < head_dim; d++) {
        float acc = 0.0f;
        for (int j = 0; j < seq_len; j++) acc += scores[j] * vbase[(size_t)j * stride + d];
        y[d] = acc;
    }
    return ORC_OK;
}

static void orc_norm(int hidden, float* y, const float* x, const float* w, float eps) {
    orc_rms_norm_f32((size_t)hidden, x, w, y, eps);
}

int orc_runner_run(const orc_runner_cfg* c, const orc_model* m, int n_tokens,
                   const int32_t* tokens, float* logits) {
    if (!c || !m || !tokens || !logits || !m->embed) return ORC_ERR_INVALID_ARG;
    const int H = c->hidden, Hq = c->n_heads, Hkv = c->n_kv_heads, d = c->head_dim;
    const int I = c->intermediate, V = c->vocab, L = c->layers, S = c->max_seq;
    if (H <= 0 || Hq <= 0 || Hkv <= 0 || d <= 0 || V <= 0 || L < 0 || S <= 0 || Hq % Hkv)
        return ORC_ERR_INVALID_ARG;
    if (n_tokens > S) return ORC_ERR_INVALID_ARG;
    const int q_dim = Hq * d, kv_dim = Hkv * d, n_rep = Hq / Hkv;
    const size_t xlen = (size_t)(H > V ? H : V);

    float* x = calloc(xlen, sizeof(float));
    float* q = calloc((size_t)q_dim, sizeof(float));
    float* k = calloc((size_t)kv_dim, sizeof(float));
    float* v = calloc((size_t)kv_dim, sizeof(float));
    float* attn = calloc((size_t)q_dim, sizeof(float));
    float* proj = calloc((size_t)H, sizeof(float));
    float* xm = calloc((size_t)H, sizeof(float));
    float* g = calloc((size_t)(I > 0 ? I : 1), sizeof(float));
    float* u = calloc((size_t)(I > 0 ? I : 1), sizeof(float));
    float* scores = calloc((size_t)S, sizeof(float));
    float* kc = calloc((size_t)L * S * kv_dim + 1, sizeof(float));
    float* vc = calloc((size_t)L * S * kv_dim + 1, sizeof(float));
    float* lg = calloc((size_t)V, sizeof(float));
    int rc = ORC_OK;
    if (!x || !q || !k || !v || !attn || !proj || !xm || !g || !u || !scores || !kc || !vc || !lg) {
        rc = ORC_ERR_OOM;
        goto done;
    }
    const float scale = 1.f / sqrtf((float)d);
    for (int t = 0; t < n_tokens; t++) {
        const int pos = t, cur = pos + 1;
        const int tok = tokens[t];
        if (tok < 0 || tok >= V) {
            rc = ORC_ERR_INVALID_ARG;
            goto done;
        }
        orc_embedding_f32(&tok, 1, H, m->embed, x);
        for (int l = 0; l < L; l++) {
            const orc_layer* ly = &m->layers[l];
            if (!ly->q.w || !ly->k.w || !ly->v.w) continue;  /* ops.hpp:109 */
            orc_norm(H, x, x, ly->in_norm, c->norm_eps);
            orc_project(&ly->q, x, q);
            orc_project(&ly->k, x, k);
            orc_project(&ly->v, x, v);
            orc_rope_gqa_f32(Hq, Hkv, d, q, k, pos, c->rope_theta);
            float* kcl = kc + (size_t)l * S * kv_dim;
            float* vcl = vc + (size_t)l * S * kv_dim;
            memcpy(kcl + (size_t)pos * kv_dim, k, (size_t)kv_dim * sizeof(float));
            memcpy(vcl + (size_t)pos * kv_dim, v, (size_t)kv_dim * sizeof(float));
            for (int r = 0; r < Hq; r++) {
                int h, last, seq;
                if (c->attention == ORC_ATTN_REFERENCE) {
                    h = r / cur;
                    last = r % cur;
                    seq = cur;
                } else {
                    h = r;
                    last = pos;
                    seq = cur;
                }
                const int gkv = h / n_rep;
                orc_attention_row(q + (size_t)h * d, kcl + (size_t)gkv * d, vcl + (size_t)gkv * d,
                                  (size_t)kv_dim, seq, last, d, scale, scores,
                                  attn + (size_t)r * d);
            }
            if (ly->o.w) {  /* :207-218 */
                orc_project(&ly->o, attn, proj);
                orc_residual_add_f32((size_t)H, proj, x, x);
            }
            orc_norm(H, xm, x, ly->post_norm, c->norm_eps);
            if (ly->gate.w && ly->up.w && I > 0) {  /* :226-256 */
                orc_project(&ly->gate, xm, g);
                orc_project(&ly->up, xm, u);
                orc_silu_f32((size_t)I, g, g);
                for (int i = 0; i < I; i++) g[i] *= u[i];
                if (ly->down.w) {
                    orc_project(&ly->down, g, proj);
                    orc_residual_add_f32((size_t)H, proj, x, x);
                }
            }
        }
        orc_norm(H, x, x, m->final_norm, c->norm_eps);  /* :260-266 */
        const float* wlm = m->lm_head ? m->lm_head : m->embed;  /* :269-273 */
        orc_dense_linear_f32((size_t)V, (size_t)H, x, wlm, NULL, lg);
        memcpy(x, lg, (size_t)V * sizeof(float));
        memcpy(logits + (size_t)t * V, lg, (size_t)V * sizeof(float));
    }
done:
    free(x), free(q), free(k), free(v), free(attn), free(proj), free(xm), free(g), free(u);
    free(scores), free(kc), free(vc), free(lg);
    return rc;
}
