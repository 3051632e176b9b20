/*
 * backend_b200.c -- the "b200" TbBackend: TbOpFn adapters that unpack
 * TbTensor arguments and call the sm_100a kernels of libtb_b200.so (C11).
 *
 * Each adapter follows the input packing of the engine's dispatch helpers
 * (src/backend/cpu/registry.c:90-201) and the argument meaning of the CPU
 * adapters (src/backend/cpu/{norm,residual,activation,rope,softmax,
 * embedding}.c), with these rules:
 *   - device tensors only: a host tensor (device != TB_DEVICE_CUDA) returns
 *     TB_ERR_INVALID_ARG.  There is no CPU fallback inside this backend;
 *   - dtypes F32 and BF16, every tensor of one call in the same dtype;
 *   - rows: a rank-1 tensor is one row (what the CPU adapters do with every
 *     tensor, e.g. cpu/norm.c:12); a tensor of rank >= 2 is
 *     [product of the leading dims, last dim], one row per leading index;
 *   - shapes are checked (TB_ERR_INVALID_SHAPE) where the CPU adapters
 *     would read or write out of bounds;
 *   - results are queued on the library's current stream
 *     (tb_b200_set_stream) and are not synchronised.
 */
#include <math.h>
#include <pthread.h>
#include <string.h>

#include "../../include/tb_b200.h"
#include "../../include/tb_backend.h"

/* ------------------------------------------------------------ helpers */

static int64_t nelem(const TbTensor* t) {
    int64_t n = 1;
    for (int i = 0; i < t->rank; i++) n *= (int64_t)t->shape[i];
    return n;
}

static void rows_cols(const TbTensor* t, int64_t* rows, int64_t* cols) {
    if (t->rank == 0) {
        *rows = 1;
        *cols = 1;
        return;
    }
    *cols = (int64_t)t->shape[t->rank - 1];
    *rows = *cols ? nelem(t) / *cols : 0;
}

static int is_dev(const TbTensor* t) { return t != NULL && t->device == TB_DEVICE_CUDA; }

static int dtype_ok(TbDtype d) { return d == TB_DTYPE_F32 || d == TB_DTYPE_BF16; }

/* All non-NULL tensors on the device, in one supported dtype. */
static int check(int n, const TbTensor* const* ts) {
    TbDtype d = TB_DTYPE_F32;
    int seen = 0;
    for (int i = 0; i < n; i++) {
        const TbTensor* t = ts[i];
        if (t == NULL) continue;
        if (!is_dev(t)) return TB_ERR_INVALID_ARG;
        if (!dtype_ok(t->dtype)) return TB_ERR_UNSUPPORTED_DTYPE;
        if (seen && t->dtype != d) return TB_ERR_UNSUPPORTED_DTYPE;
        d = t->dtype;
        seen = 1;
    }
    return TB_OK;
}

#define IN(i) ((n_inputs > (i)) ? (const TbTensor*)inputs[(i)] : NULL)

/* --------------------------------------------------------------- ops */

/* SPARSE_LINEAR: inputs {x, w, mask, bias}, params N:M (defaults 2:4 as in
 * src/backend/cpu/linear.c:16-24); out = w.shape[0], in = w.shape[1].  f32
 * vectors and weights, a U8 device mask. */
static int b200_sparse_linear(void* output, const void** inputs, int n_inputs,
                              const void* params) {
    TbTensor* y = (TbTensor*)output;
    const TbTensor* x = IN(0);
    const TbTensor* w = IN(1);
    const TbTensor* mask = IN(2);
    const TbTensor* bias = IN(3);
    if (!x || !w || !mask || !y || w->rank < 2) return TB_ERR_INVALID_ARG;
    const TbTensor* ts[] = {y, x, w, bias};
    int rc = check(4, ts);
    if (rc) return rc;
    if (x->dtype != TB_DTYPE_F32) return TB_ERR_UNSUPPORTED_DTYPE;
    if (!is_dev(mask)) return TB_ERR_INVALID_ARG;
    if (mask->dtype != TB_DTYPE_U8) return TB_ERR_UNSUPPORTED_DTYPE;
    int nm_n = 2, nm_m = 4;
    if (params) {
        const TbLinearParams* lp = (const TbLinearParams*)params;
        nm_n = lp->nm_n > 0 ? lp->nm_n : 2;
        nm_m = lp->nm_m > 0 ? lp->nm_m : 4;
    }
    const int64_t out_f = (int64_t)w->shape[0], in_f = (int64_t)w->shape[1];
    if (nelem(x) < in_f || nelem(y) < out_f || (bias && nelem(bias) < out_f) ||
        (nm_m >= 2 && nelem(mask) < out_f * (in_f / nm_m)))
        return TB_ERR_INVALID_SHAPE;
    return tb_b200_sparse_linear(out_f, in_f, (const float*)x->data, (const float*)w->data,
                                 (const uint8_t*)mask->data,
                                 bias ? (const float*)bias->data : NULL, (float*)y->data, nm_n,
                                 nm_m, NULL);
}

/* DENSE_LINEAR: inputs {x, w, bias}; out = nelem(y) (the CPU adapter's rule
 * for tied embeddings, src/backend/cpu/linear.c:38-44), in = w.shape[1]. */
static int b200_dense_linear(void* output, const void** inputs, int n_inputs,
                             const void* params) {
    (void)params;
    TbTensor* y = (TbTensor*)output;
    const TbTensor* x = IN(0);
    const TbTensor* w = IN(1);
    const TbTensor* bias = IN(2);
    if (!x || !w || !y || w->rank < 2) return TB_ERR_INVALID_ARG;
    const TbTensor* ts[] = {y, x, w, bias};
    int rc = check(4, ts);
    if (rc) return rc;
    if (x->dtype != TB_DTYPE_F32) return TB_ERR_UNSUPPORTED_DTYPE;
    const int64_t out_f = nelem(y), in_f = (int64_t)w->shape[1];
    if (nelem(x) < in_f || out_f > (int64_t)w->shape[0] || (bias && nelem(bias) < out_f))
        return TB_ERR_INVALID_SHAPE;
    return tb_b200_dense_linear(out_f, in_f, (const float*)x->data, (const float*)w->data,
                                bias ? (const float*)bias->data : NULL, (float*)y->data, NULL);
}

/* RMS_NORM: inputs {x, weight}, params TbNormParams (eps defaults to 1e-6f
 * as in src/backend/cpu/norm.c:6). */
static int b200_rms_norm(void* output, const void** inputs, int n_inputs, const void* params) {
    TbTensor* y = (TbTensor*)output;
    const TbTensor* x = IN(0);
    const TbTensor* w = IN(1);
    if (!x || !y) return TB_ERR_INVALID_ARG;
    const TbTensor* ts[] = {y, x, w};
    int rc = check(3, ts);
    if (rc) return rc;
    const float eps = params ? ((const TbNormParams*)params)->eps : 1e-6f;
    int64_t rows, cols;
    rows_cols(x, &rows, &cols);
    if (nelem(y) != nelem(x) || (w && nelem(w) != cols)) return TB_ERR_INVALID_SHAPE;
    return tb_b200_rms_norm(x->dtype, rows, cols, x->data, w ? w->data : NULL, y->data, eps, NULL);
}

/* RESIDUAL_ADD: inputs {x, residual}. */
static int b200_residual_add(void* output, const void** inputs, int n_inputs,
                             const void* params) {
    (void)params;
    TbTensor* y = (TbTensor*)output;
    const TbTensor* x = IN(0);
    const TbTensor* r = IN(1);
    if (!x || !r || !y) return TB_ERR_INVALID_ARG;
    const TbTensor* ts[] = {y, x, r};
    int rc = check(3, ts);
    if (rc) return rc;
    if (nelem(y) != nelem(x) || nelem(r) != nelem(x)) return TB_ERR_INVALID_SHAPE;
    return tb_b200_residual_add(x->dtype, nelem(x), x->data, r->data, y->data, NULL);
}

static int unary(int which, void* output, const void** inputs, int n_inputs) {
    TbTensor* y = (TbTensor*)output;
    const TbTensor* x = IN(0);
    if (!x || !y) return TB_ERR_INVALID_ARG;
    const TbTensor* ts[] = {y, x};
    int rc = check(2, ts);
    if (rc) return rc;
    if (nelem(y) != nelem(x)) return TB_ERR_INVALID_SHAPE;
    if (which == 0) return tb_b200_gelu(x->dtype, nelem(x), x->data, y->data, NULL);
    return tb_b200_silu(x->dtype, nelem(x), x->data, y->data, NULL);
}

/* GELU / SILU: inputs {x}. */
static int b200_gelu(void* output, const void** inputs, int n_inputs, const void* params) {
    (void)params;
    return unary(0, output, inputs, n_inputs);
}

static int b200_silu(void* output, const void** inputs, int n_inputs, const void* params) {
    (void)params;
    return unary(1, output, inputs, n_inputs);
}

/* SOFTMAX: inputs {x, mask}; mask optional, same shape as x. */
static int b200_softmax(void* output, const void** inputs, int n_inputs, const void* params) {
    (void)params;
    TbTensor* y = (TbTensor*)output;
    const TbTensor* x = IN(0);
    const TbTensor* m = IN(1);
    if (!x || !y) return TB_ERR_INVALID_ARG;
    const TbTensor* ts[] = {y, x, m};
    int rc = check(3, ts);
    if (rc) return rc;
    if (nelem(y) != nelem(x) || (m && nelem(m) != nelem(x))) return TB_ERR_INVALID_SHAPE;
    int64_t rows, cols;
    rows_cols(x, &rows, &cols);
    return tb_b200_softmax(x->dtype, rows, cols, x->data, m ? m->data : NULL, y->data, NULL);
}

/* ROPE: output q, inputs {k}, params TbRopeParams.  As in
 * src/backend/cpu/rope.c:11-13, the head counts are q/k shape[0] and
 * head_dim is q's last dimension (shape[2] of the engine's [heads, 1, d]). */
static int b200_rope(void* output, const void** inputs, int n_inputs, const void* params) {
    TbTensor* q = (TbTensor*)output;
    const TbTensor* k = IN(0);
    const TbRopeParams* p = (const TbRopeParams*)params;
    if (!q || !k || !p) return TB_ERR_INVALID_ARG;
    const TbTensor* ts[] = {q, k};
    int rc = check(2, ts);
    if (rc) return rc;
    if (q->rank < 2 || k->rank < 2) return TB_ERR_INVALID_SHAPE;
    const int hq = (int)q->shape[0], hkv = (int)k->shape[0];
    const int d = (int)q->shape[q->rank - 1];
    if ((int)k->shape[k->rank - 1] != d || nelem(q) != (int64_t)hq * d ||
        nelem(k) != (int64_t)hkv * d)
        return TB_ERR_INVALID_SHAPE;
    return tb_b200_rope(q->dtype, hq, hkv, d, q->data, k->data, p->position, p->theta, NULL);
}

/* EMBEDDING: inputs {const int* ids, const int* n_tokens, table}
 * (src/backend/cpu/embedding.c:7-9); ids may be host or device memory. */
static int b200_embedding(void* output, const void** inputs, int n_inputs, const void* params) {
    (void)params;
    TbTensor* y = (TbTensor*)output;
    if (n_inputs < 3 || !y) return TB_ERR_INVALID_ARG;
    const int32_t* ids = (const int32_t*)inputs[0];
    const int n_tokens = inputs[1] ? *(const int*)inputs[1] : 1;
    const TbTensor* table = (const TbTensor*)inputs[2];
    if (!ids || !table) return TB_ERR_INVALID_ARG;
    const TbTensor* ts[] = {y, table};
    int rc = check(2, ts);
    if (rc) return rc;
    if (table->rank != 2 || n_tokens < 0) return TB_ERR_INVALID_SHAPE;
    const int64_t vocab = (int64_t)table->shape[0], dim = (int64_t)table->shape[1];
    if (nelem(y) < (int64_t)n_tokens * dim) return TB_ERR_INVALID_SHAPE;
    int on_dev = 0;
    rc = tb_b200_is_device_ptr(ids, &on_dev);
    if (rc) return rc;
    if (on_dev)
        return tb_b200_embedding(table->dtype, n_tokens, dim, vocab, ids, table->data, y->data,
                                 NULL);
    return tb_b200_embedding_host_ids(table->dtype, n_tokens, dim, vocab, ids, table->data,
                                      y->data, NULL);
}

/* RESIDUAL_RMS_NORM: inputs {x, residual, weight, h_out}. */
static int b200_residual_rms_norm(void* output, const void** inputs, int n_inputs,
                                  const void* params) {
    TbTensor* y = (TbTensor*)output;
    const TbTensor* x = IN(0);
    const TbTensor* r = IN(1);
    const TbTensor* w = IN(2);
    TbTensor* h = (TbTensor*)IN(3);
    if (!x || !y) return TB_ERR_INVALID_ARG;
    const TbTensor* ts[] = {y, x, r, w, h};
    int rc = check(5, ts);
    if (rc) return rc;
    const float eps = params ? ((const TbNormParams*)params)->eps : 1e-6f;
    int64_t rows, cols;
    rows_cols(x, &rows, &cols);
    if (nelem(y) != nelem(x) || (r && nelem(r) != nelem(x)) || (h && nelem(h) != nelem(x)) ||
        (w && nelem(w) != cols))
        return TB_ERR_INVALID_SHAPE;
    return tb_b200_residual_rms_norm(x->dtype, rows, cols, x->data, r ? r->data : NULL,
                                     w ? w->data : NULL, h ? h->data : NULL, y->data, eps, NULL);
}

/* SWIGLU: inputs {gate, up}. */
static int b200_swiglu(void* output, const void** inputs, int n_inputs, const void* params) {
    (void)params;
    TbTensor* out = (TbTensor*)output;
    const TbTensor* g = IN(0);
    const TbTensor* u = IN(1);
    if (!out || !g || !u) return TB_ERR_INVALID_ARG;
    const TbTensor* ts[] = {out, g, u};
    int rc = check(3, ts);
    if (rc) return rc;
    if (nelem(out) != nelem(g) || nelem(u) != nelem(g)) return TB_ERR_INVALID_SHAPE;
    return tb_b200_swiglu(g->dtype, nelem(g), g->data, u->data, out->data, NULL);
}

/* ARGMAX: output I32 [rows], inputs {logits}. */
static int b200_argmax(void* output, const void** inputs, int n_inputs, const void* params) {
    (void)params;
    TbTensor* out = (TbTensor*)output;
    const TbTensor* x = IN(0);
    if (!out || !x) return TB_ERR_INVALID_ARG;
    const TbTensor* ts[] = {x};
    int rc = check(1, ts);
    if (rc) return rc;
    if (!is_dev(out)) return TB_ERR_INVALID_ARG;
    if (out->dtype != TB_DTYPE_I32) return TB_ERR_UNSUPPORTED_DTYPE;
    int64_t rows, cols;
    rows_cols(x, &rows, &cols);
    if (nelem(out) != rows) return TB_ERR_INVALID_SHAPE;
    return tb_b200_argmax(x->dtype, rows, cols, x->data, (int32_t*)out->data, NULL);
}

/* ---- cached cos/sin tables for TB_OP_ROPE_ROWS, per (device, theta, d) */

typedef struct {
    int device, head_dim, n_positions;
    float theta;
    float* table;
} RopeTable;

#define ROPE_CACHE 16
static RopeTable g_rope[ROPE_CACHE];
static pthread_mutex_t g_rope_mu = PTHREAD_MUTEX_INITIALIZER;

/* A device table covering at least `max_position` positions, or NULL when
 * max_position is 0 (then every row computes cos/sin on the device). */
static int rope_table_for(float theta, int head_dim, int max_position, const float** out,
                          int* n_out) {
    *out = NULL;
    *n_out = 0;
    if (max_position <= 0) return TB_OK;
    int dev = 0;
    int rc = tb_b200_get_device(&dev);
    if (rc) return rc;
    pthread_mutex_lock(&g_rope_mu);
    RopeTable* slot = NULL;
    for (int i = 0; i < ROPE_CACHE; i++) {
        RopeTable* t = &g_rope[i];
        if (t->table && t->device == dev && t->head_dim == head_dim && t->theta == theta) {
            slot = t;
            break;
        }
    }
    if (slot && slot->n_positions < max_position) {
        tb_b200_free(slot->table);
        slot->table = NULL;
    }
    if (!slot) {
        for (int i = 0; i < ROPE_CACHE && !slot; i++)
            if (!g_rope[i].table) slot = &g_rope[i];
        if (!slot) { /* full: recycle the first entry */
            slot = &g_rope[0];
            tb_b200_free(slot->table);
            slot->table = NULL;
        }
    }
    if (!slot->table) {
        void* p = NULL;
        rc = tb_b200_malloc(&p, (size_t)max_position * (size_t)head_dim * sizeof(float));
        if (rc == TB_OK) rc = tb_b200_rope_table(theta, head_dim, max_position, (float*)p, NULL);
        if (rc) {
            tb_b200_free(p);
            pthread_mutex_unlock(&g_rope_mu);
            return rc;
        }
        slot->table = (float*)p;
        slot->device = dev;
        slot->head_dim = head_dim;
        slot->theta = theta;
        slot->n_positions = max_position;
    }
    *out = slot->table;
    *n_out = slot->n_positions;
    pthread_mutex_unlock(&g_rope_mu);
    return TB_OK;
}

/* Device copy of `positions` when they are host memory. */
static int positions_on_device(const int32_t* pos, int64_t rows, const int32_t** dev,
                               void** staged) {
    *staged = NULL;
    int on_dev = 0;
    int rc = tb_b200_is_device_ptr(pos, &on_dev);
    if (rc) return rc;
    if (on_dev) {
        *dev = pos;
        return TB_OK;
    }
    rc = tb_b200_stage_h2d(pos, (size_t)rows * sizeof(int32_t), staged, NULL);
    *dev = (const int32_t*)*staged;
    return rc;
}

/* ROPE_ROWS: output q [rows, hq, d], inputs {k [rows, hkv, d]},
 * params TbRopeRowsParams. */
static int b200_rope_rows(void* output, const void** inputs, int n_inputs, const void* params) {
    TbTensor* q = (TbTensor*)output;
    const TbTensor* k = IN(0);
    const TbRopeRowsParams* p = (const TbRopeRowsParams*)params;
    if (!q || !k || !p || !p->positions) return TB_ERR_INVALID_ARG;
    const TbTensor* ts[] = {q, k};
    int rc = check(2, ts);
    if (rc) return rc;
    if (q->rank != 3 || k->rank != 3 || q->shape[0] != k->shape[0] || q->shape[2] != k->shape[2])
        return TB_ERR_INVALID_SHAPE;
    const int64_t rows = (int64_t)q->shape[0];
    const int d = (int)q->shape[2];
    if (p->head_dim > 0 && p->head_dim != d) return TB_ERR_INVALID_SHAPE;
    const float* table;
    int npos;
    rc = rope_table_for(p->theta, d, p->max_position, &table, &npos);
    if (rc) return rc;
    const int32_t* pos;
    void* staged;
    rc = positions_on_device(p->positions, rows, &pos, &staged);
    if (rc) return rc;
    rc = tb_b200_rope_rows(q->dtype, rows, (int)q->shape[1], (int)k->shape[1], d, q->data, k->data,
                           pos, p->theta, table, npos, NULL);
    const int rc2 = tb_b200_stage_release(staged, NULL);
    return rc ? rc : rc2;
}

/* LAYER_CHAIN: output y, inputs {h_out, act, x, residual, weight, q, k,
 * gate, up}, params TbLayerChainParams. */
static int b200_layer_chain(void* output, const void** inputs, int n_inputs, const void* params) {
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
    int rc = check(10, ts);
    if (rc) return rc;
    TbB200LayerChain c;
    memset(&c, 0, sizeof c);
    c.dtype = x->dtype;
    int64_t rows, hidden;
    rows_cols(x, &rows, &hidden);
    c.rows = rows;
    c.hidden = hidden;
    c.x = x->data;
    c.residual = r ? r->data : NULL;
    c.norm_weight = w ? w->data : NULL;
    c.h_out = h ? h->data : NULL;
    c.y = y->data;
    c.eps = p->eps;
    if (nelem(y) != nelem(x) || (r && nelem(r) != nelem(x)) || (h && nelem(h) != nelem(x)) ||
        (w && nelem(w) != hidden))
        return TB_ERR_INVALID_SHAPE;
    void* staged = NULL;
    if (q && k) {
        if (q->rank != 3 || k->rank != 3 || (int64_t)q->shape[0] != rows ||
            (int64_t)k->shape[0] != rows || q->shape[2] != k->shape[2] || !p->positions)
            return TB_ERR_INVALID_SHAPE;
        c.n_q_heads = (int)q->shape[1];
        c.n_kv_heads = (int)k->shape[1];
        c.head_dim = (int)q->shape[2];
        c.q = q->data;
        c.k = k->data;
        c.theta = p->theta;
        rc = rope_table_for(p->theta, c.head_dim, p->max_position, &c.rope_table,
                            &c.rope_table_positions);
        if (rc) return rc;
        rc = positions_on_device(p->positions, rows, &c.positions, &staged);
        if (rc) return rc;
    }
    if (g && u && act) {
        int64_t grow, inter;
        rows_cols(g, &grow, &inter);
        if (grow != rows || nelem(u) != nelem(g) || nelem(act) != nelem(g)) {
            tb_b200_stage_release(staged, NULL);
            return TB_ERR_INVALID_SHAPE;
        }
        c.intermediate = inter;
        c.gate = g->data;
        c.up = u->data;
        c.act_out = act->data;
    }
    rc = tb_b200_layer_chain(&c, NULL);
    const int rc2 = tb_b200_stage_release(staged, NULL);
    return rc ? rc : rc2;
}

/* ---------------------------------------------------------- register */

static int g_b200_registered = 0;

int tb_backend_b200_init(void) {
    if (g_b200_registered) {
        for (int i = 0; i < tb_backend_count(); i++) {
            const TbBackend* be = tb_backend_get(i);
            if (be && be->name && strcmp(be->name, "b200") == 0) return TB_OK;
        }
    }
    TbBackend be;
    memset(&be, 0, sizeof be);
    be.name = "b200";
    be.priority = 200;
    be.ops[TB_OP_SPARSE_LINEAR] = b200_sparse_linear;
    be.ops[TB_OP_DENSE_LINEAR] = b200_dense_linear;
    be.ops[TB_OP_RMS_NORM] = b200_rms_norm;
    be.ops[TB_OP_RESIDUAL_ADD] = b200_residual_add;
    be.ops[TB_OP_GELU] = b200_gelu;
    be.ops[TB_OP_SILU] = b200_silu;
    be.ops[TB_OP_SOFTMAX] = b200_softmax;
    be.ops[TB_OP_ROPE] = b200_rope;
    be.ops[TB_OP_EMBEDDING] = b200_embedding;
    be.ops[TB_OP_RESIDUAL_RMS_NORM] = b200_residual_rms_norm;
    be.ops[TB_OP_SWIGLU] = b200_swiglu;
    be.ops[TB_OP_ARGMAX] = b200_argmax;
    be.ops[TB_OP_ROPE_ROWS] = b200_rope_rows;
    be.ops[TB_OP_LAYER_CHAIN] = b200_layer_chain;
    const int rc = tb_backend_register_device(&be, TB_DEVICE_CUDA);
    if (rc == TB_OK) g_b200_registered = 1;
    return rc;
}
