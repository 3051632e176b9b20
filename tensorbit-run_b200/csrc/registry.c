/*
 * registry.c -- tensorbit-run's backend registry and tb_dispatch_* helpers,
 * with device-aware routing (C11).
 *
 * Behaviour kept from the engine's registry (src/backend/cpu/registry.c):
 *   - a static table of at most TB_MAX_BACKENDS vtables, copied on
 *     registration; registering past the limit returns -1 (registry.c:28-35);
 *   - tb_backend_get_best(op) returns the highest-priority backend whose slot
 *     for `op` is non-NULL, over every registered backend (registry.c:37-50);
 *   - each tb_dispatch_* packs `inputs` and a parameter struct exactly as
 *     the engine does and calls the chosen slot (registry.c:90-201); no
 *     backend found returns TB_ERR_BACKEND_NOT_FOUND.
 * Added: a backend may be registered for one device
 * (tb_backend_register_device); tb_dispatch_* choose among the backends that
 * serve the device of the first tensor argument, so a "b200" backend
 * registered for TB_DEVICE_CUDA never receives host tensors and host
 * tensors keep reaching "cpu".  Like the engine's, the registry is not
 * synchronised: register backends before dispatching from several threads.
 */
#include <string.h>

#include "../../include/tb_backend.h"

typedef struct {
    TbBackend be;
    int device; /* a TbDevice, or -1 for every device */
} TbEntry;

static TbEntry g_entries[TB_MAX_BACKENDS];
static int g_count = 0;

static int register_entry(const TbBackend* backend, int device) {
    if (backend == NULL) return TB_ERR_INVALID_ARG;
    if (g_count >= TB_MAX_BACKENDS) return -1;
    g_entries[g_count].be = *backend;
    g_entries[g_count].device = device;
    g_count++;
    return TB_OK;
}

int tb_backend_register(const TbBackend* backend) { return register_entry(backend, -1); }

int tb_backend_register_device(const TbBackend* backend, TbDevice device) {
    return register_entry(backend, (int)device);
}

void tb_backend_reset(void) {
    memset(g_entries, 0, sizeof g_entries);
    g_count = 0;
}

static const TbBackend* best(TbOpType op, int device) {
    if ((int)op < 0 || op >= TB_OP_COUNT) return NULL;
    const TbBackend* found = NULL;
    int prio = -1;
    for (int i = 0; i < g_count; i++) {
        const TbEntry* e = &g_entries[i];
        if (e->be.ops[op] == NULL) continue;
        if (device >= 0 && e->device >= 0 && e->device != device) continue;
        if (e->be.priority > prio) {
            prio = e->be.priority;
            found = &e->be;
        }
    }
    return found;
}

const TbBackend* tb_backend_get_best(TbOpType op) { return best(op, -1); }

const TbBackend* tb_backend_get_best_device(TbOpType op, TbDevice device) {
    return best(op, (int)device);
}

int tb_backend_count(void) { return g_count; }

const TbBackend* tb_backend_get(int index) {
    if (index < 0 || index >= g_count) return NULL;
    return &g_entries[index].be;
}

/* ------------------------------------------------------------- dispatch */

static int dev_of(const TbTensor* t) { return t ? (int)t->device : (int)TB_DEVICE_CPU; }

#define PICK(op, t)                                              \
    const TbBackend* be = best((op), dev_of(t));                 \
    if (be == NULL) return TB_ERR_BACKEND_NOT_FOUND

int tb_dispatch_sparse_linear(TbTensor* y, const TbTensor* x, const TbTensor* w,
                              const TbTensor* mask, const TbTensor* bias) {
    PICK(TB_OP_SPARSE_LINEAR, y);
    const void* arr[] = {x, w, mask, bias};
    return be->ops[TB_OP_SPARSE_LINEAR](y, arr, 4, NULL);
}

int tb_dispatch_dense_linear(TbTensor* y, const TbTensor* x, const TbTensor* w,
                             const TbTensor* bias) {
    PICK(TB_OP_DENSE_LINEAR, y);
    const void* arr[] = {x, w, bias};
    return be->ops[TB_OP_DENSE_LINEAR](y, arr, 3, NULL);
}

int tb_dispatch_rms_norm(TbTensor* y, const TbTensor* x, const TbTensor* weight, float eps) {
    PICK(TB_OP_RMS_NORM, y);
    TbNormParams p = {eps};
    const void* arr[] = {x, weight};
    return be->ops[TB_OP_RMS_NORM](y, arr, 2, &p);
}

int tb_dispatch_layer_norm(TbTensor* y, const TbTensor* x, const TbTensor* weight,
                           const TbTensor* bias, float eps) {
    PICK(TB_OP_LAYER_NORM, y);
    TbNormParams p = {eps};
    const void* arr[] = {x, weight, bias};
    return be->ops[TB_OP_LAYER_NORM](y, arr, 3, &p);
}

int tb_dispatch_gelu(TbTensor* y, const TbTensor* x) {
    PICK(TB_OP_GELU, y);
    const void* arr[] = {x};
    return be->ops[TB_OP_GELU](y, arr, 1, NULL);
}

int tb_dispatch_silu(TbTensor* y, const TbTensor* x) {
    PICK(TB_OP_SILU, y);
    const void* arr[] = {x};
    return be->ops[TB_OP_SILU](y, arr, 1, NULL);
}

int tb_dispatch_softmax(TbTensor* y, const TbTensor* x, const TbTensor* mask) {
    PICK(TB_OP_SOFTMAX, y);
    const void* arr[] = {x, mask};
    return be->ops[TB_OP_SOFTMAX](y, arr, 2, NULL);
}

/* The engine's QKV helper is three sparse_linear dispatches
 * (src/backend/cpu/registry.c:144-159); kept as is. */
int tb_dispatch_attention_qkv(TbTensor* q, TbTensor* k, TbTensor* v, const TbTensor* x,
                              const TbTensor* wq, const TbTensor* wk, const TbTensor* wv,
                              const TbTensor* mq, const TbTensor* mk, const TbTensor* mv,
                              int num_heads, int num_kv_heads, int head_dim) {
    int ret = tb_dispatch_sparse_linear(q, x, wq, mq, NULL);
    if (ret) return ret;
    ret = tb_dispatch_sparse_linear(k, x, wk, mk, NULL);
    if (ret) return ret;
    ret = tb_dispatch_sparse_linear(v, x, wv, mv, NULL);
    if (ret) return ret;
    (void)num_heads;
    (void)num_kv_heads;
    (void)head_dim;
    return TB_OK;
}

int tb_dispatch_scaled_dot_product(TbTensor* y, const TbTensor* q, const TbTensor* k,
                                   const TbTensor* v, const TbTensor* mask, float scale,
                                   bool causal) {
    PICK(TB_OP_SCALED_DOT_PRODUCT, y);
    TbSdpParams p = {scale, causal, 0};
    const void* arr[] = {q, k, v, mask};
    return be->ops[TB_OP_SCALED_DOT_PRODUCT](y, arr, 4, &p);
}

int tb_dispatch_rope(TbTensor* q, TbTensor* k, int position, float theta, int head_dim) {
    PICK(TB_OP_ROPE, q);
    TbRopeParams p = {position, theta, head_dim};
    const void* arr[] = {k};
    return be->ops[TB_OP_ROPE](q, arr, 1, &p);
}

int tb_dispatch_residual_add(TbTensor* y, const TbTensor* x, const TbTensor* residual) {
    PICK(TB_OP_RESIDUAL_ADD, y);
    const void* arr[] = {x, residual};
    return be->ops[TB_OP_RESIDUAL_ADD](y, arr, 2, NULL);
}

int tb_dispatch_embedding(TbTensor* y, const int* token_ids, int n_tokens,
                          const TbTensor* embedding) {
    PICK(TB_OP_EMBEDDING, y);
    const void* arr[] = {token_ids, &n_tokens, embedding};
    return be->ops[TB_OP_EMBEDDING](y, arr, 3, NULL);
}

int tb_dispatch_conv2d(TbTensor* y, const TbTensor* x, const TbTensor* kernel,
                       const TbTensor* bias, int stride, int padding) {
    PICK(TB_OP_CONV2D, y);
    TbConv2dParams p = {stride, padding};
    const void* arr[] = {x, kernel, bias};
    return be->ops[TB_OP_CONV2D](y, arr, 3, &p);
}

/* ----------------------------------------------------- added operations */

int tb_dispatch_residual_rms_norm(TbTensor* y, TbTensor* h_out, const TbTensor* x,
                                  const TbTensor* residual, const TbTensor* weight, float eps) {
    PICK(TB_OP_RESIDUAL_RMS_NORM, y);
    TbNormParams p = {eps};
    const void* arr[] = {x, residual, weight, h_out};
    return be->ops[TB_OP_RESIDUAL_RMS_NORM](y, arr, 4, &p);
}

int tb_dispatch_swiglu(TbTensor* out, const TbTensor* gate, const TbTensor* up) {
    PICK(TB_OP_SWIGLU, out);
    const void* arr[] = {gate, up};
    return be->ops[TB_OP_SWIGLU](out, arr, 2, NULL);
}

int tb_dispatch_argmax(TbTensor* out, const TbTensor* logits) {
    PICK(TB_OP_ARGMAX, logits);
    const void* arr[] = {logits};
    return be->ops[TB_OP_ARGMAX](out, arr, 1, NULL);
}

int tb_dispatch_rope_rows(TbTensor* q, TbTensor* k, const int32_t* positions, float theta,
                          int head_dim, int max_position) {
    PICK(TB_OP_ROPE_ROWS, q);
    TbRopeRowsParams p = {positions, theta, head_dim, max_position};
    const void* arr[] = {k};
    return be->ops[TB_OP_ROPE_ROWS](q, arr, 1, &p);
}

int tb_dispatch_layer_chain(TbTensor* y, TbTensor* h_out, TbTensor* act, const TbTensor* x,
                            const TbTensor* residual, const TbTensor* weight, TbTensor* q,
                            TbTensor* k, const TbTensor* gate, const TbTensor* up,
                            const TbLayerChainParams* params) {
    PICK(TB_OP_LAYER_CHAIN, y);
    const void* arr[] = {h_out, act, x, residual, weight, q, k, gate, up};
    return be->ops[TB_OP_LAYER_CHAIN](y, arr, 9, params);
}
