/*
 * tb_backend.h -- tensorbit-run's backend registry with the b200 backend.
 *
 * This is the engine's registry API (include/tensorbit/run/backend.h) with
 * the additions the b200 backend needs, restated so the b200 library can be
 * built and tested on its own.  It is a superset: the original 13 op slots,
 * parameter structs, TbOpFn signature, TbBackend layout and every original
 * tb_dispatch_* signature are unchanged (backend.h:15-140).  Additions:
 *   - five op types appended before TB_OP_COUNT (fused and row-batched ops);
 *   - device-aware routing: a backend may be registered for one device, and
 *     tb_dispatch_* picks the best backend for the device of the tensors it
 *     is given, so host tensors keep reaching "cpu" while device tensors
 *     reach "b200" (the original tb_backend_get_best, backend.h:92, is
 *     device-blind and is kept as it was);
 *   - tb_backend_b200_init, which registers "b200" for TB_DEVICE_CUDA.
 * A build that uses this header in place of backend.h links this library's
 * registry (registry.c) instead of the registry half of
 * src/backend/cpu/registry.c; the CPU adapters (the other files of
 * src/backend/cpu/) are unaffected.  Do not include both headers in one translation unit.
 */
#ifndef TB_BACKEND_H
#define TB_BACKEND_H

#ifdef TENSORBIT_RUN_BACKEND_H
#error "tb_backend.h is the b200-extended registry API; include it instead of tensorbit/run/backend.h"
#endif

#include "tb_types.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Op slots.  0..12 are the engine's (backend.h:15-30), values unchanged. */
typedef enum {
    TB_OP_SPARSE_LINEAR = 0,
    TB_OP_DENSE_LINEAR,
    TB_OP_RMS_NORM,
    TB_OP_LAYER_NORM,
    TB_OP_GELU,
    TB_OP_SILU,
    TB_OP_SOFTMAX,
    TB_OP_ATTENTION_QKV,
    TB_OP_SCALED_DOT_PRODUCT,
    TB_OP_ROPE,
    TB_OP_RESIDUAL_ADD,
    TB_OP_EMBEDDING,
    TB_OP_CONV2D,
    /* additions */
    TB_OP_RESIDUAL_RMS_NORM, /* h = x + residual; y = rms_norm(h) (fused)   */
    TB_OP_SWIGLU,            /* out = silu(gate) * up                        */
    TB_OP_ARGMAX,            /* per-row first index of the maximum          */
    TB_OP_ROPE_ROWS,         /* RoPE of [rows, heads, d] at per-row positions */
    TB_OP_LAYER_CHAIN,       /* the three row-op groups of a layer, 1 launch */
    TB_OP_COUNT
} TbOpType;

/* Parameter structs of the engine (backend.h:36-61), unchanged. */
typedef struct {
    int num_heads;
    int num_kv_heads;
    int head_dim;
} TbQkvParams;

typedef struct {
    float eps;
} TbNormParams;

/* N:M of a sparse linear layer (include/tensorbit/run/ops.h:23-26 in the
 * engine; the CPU adapter reads it from the op's params).  In the engine,
 * ops.h is included first and its definition stands. */
#ifndef TENSORBIT_RUN_OPS_H
typedef struct {
    int nm_n;
    int nm_m;
} TbLinearParams;
#endif

typedef struct {
    float scale;
    bool causal;
    int seq_len;
} TbSdpParams;

typedef struct {
    int position;
    float theta;
    int head_dim;
} TbRopeParams;

typedef struct {
    int stride;
    int padding;
} TbConv2dParams;

/* Parameters of TB_OP_ROPE_ROWS.  positions: one int32 per row, in the same
 * memory space as q/k.  max_position: an upper bound (exclusive) on the
 * positions, used to size the backend's cached cos/sin table; 0 = unknown. */
typedef struct {
    const int32_t* positions;
    float theta;
    int head_dim;
    int max_position;
} TbRopeRowsParams;

/* Parameters of TB_OP_LAYER_CHAIN (inputs: see tb_dispatch_layer_chain). */
typedef struct {
    float eps;
    const int32_t* positions;
    float theta;
    int head_dim;
    int max_position;
} TbLayerChainParams;

/* Uniform op signature (backend.h:69). */
typedef int (*TbOpFn)(void* output, const void** inputs, int n_inputs, const void* params);

/* Backend vtable (backend.h:75-79). */
typedef struct {
    const char* name;
    int priority;
    TbOpFn ops[TB_OP_COUNT];
} TbBackend;

#define TB_MAX_BACKENDS 8

/* Registry (backend.h:86-98).  tb_backend_register registers a backend for
 * every device, as the engine's registry does. */
int tb_backend_register(const TbBackend* backend);
const TbBackend* tb_backend_get_best(TbOpType op);
int tb_backend_count(void);
const TbBackend* tb_backend_get(int index);

/* Register a backend that serves tensors of one device only. */
int tb_backend_register_device(const TbBackend* backend, TbDevice device);
/* Highest-priority backend with a slot for `op` serving `device`. */
const TbBackend* tb_backend_get_best_device(TbOpType op, TbDevice device);
/* Forget every registered backend (tests and re-initialisation). */
void tb_backend_reset(void);

/* Dispatch helpers of the engine (backend.h:104-140), same signatures; the
 * backend is chosen for the device of the first tensor argument. */
int tb_dispatch_sparse_linear(TbTensor* y, const TbTensor* x, const TbTensor* w,
                              const TbTensor* mask, const TbTensor* bias);
int tb_dispatch_dense_linear(TbTensor* y, const TbTensor* x, const TbTensor* w,
                             const TbTensor* bias);
int tb_dispatch_rms_norm(TbTensor* y, const TbTensor* x, const TbTensor* weight, float eps);
int tb_dispatch_layer_norm(TbTensor* y, const TbTensor* x, const TbTensor* weight,
                           const TbTensor* bias, float eps);
int tb_dispatch_gelu(TbTensor* y, const TbTensor* x);
int tb_dispatch_silu(TbTensor* y, const TbTensor* x);
int tb_dispatch_softmax(TbTensor* y, const TbTensor* x, const TbTensor* mask);
int tb_dispatch_attention_qkv(TbTensor* q, TbTensor* k, TbTensor* v, const TbTensor* x,
                              const TbTensor* wq, const TbTensor* wk, const TbTensor* wv,
                              const TbTensor* mq, const TbTensor* mk, const TbTensor* mv,
                              int num_heads, int num_kv_heads, int head_dim);
int tb_dispatch_scaled_dot_product(TbTensor* y, const TbTensor* q, const TbTensor* k,
                                   const TbTensor* v, const TbTensor* mask, float scale,
                                   bool causal);
int tb_dispatch_rope(TbTensor* q, TbTensor* k, int position, float theta, int head_dim);
int tb_dispatch_residual_add(TbTensor* y, const TbTensor* x, const TbTensor* residual);
int tb_dispatch_embedding(TbTensor* y, const int* token_ids, int n_tokens,
                          const TbTensor* embedding);
int tb_dispatch_conv2d(TbTensor* y, const TbTensor* x, const TbTensor* kernel,
                       const TbTensor* bias, int stride, int padding);

/* Dispatch helpers of the added ops.  Tensors of rank >= 2 are
 * [rows = product of leading dims, cols = last dim]; rank 1 is one row. */
int tb_dispatch_residual_rms_norm(TbTensor* y, TbTensor* h_out, const TbTensor* x,
                                  const TbTensor* residual, const TbTensor* weight, float eps);
int tb_dispatch_swiglu(TbTensor* out, const TbTensor* gate, const TbTensor* up);
/* out: I32 tensor with one element per row of logits. */
int tb_dispatch_argmax(TbTensor* out, const TbTensor* logits);
/* q [rows, n_q_heads, head_dim], k [rows, n_kv_heads, head_dim], in place. */
int tb_dispatch_rope_rows(TbTensor* q, TbTensor* k, const int32_t* positions, float theta,
                          int head_dim, int max_position);
/* Inputs: x, residual, norm weight, q, k, gate, up; outputs: y, h_out, act. */
int tb_dispatch_layer_chain(TbTensor* y, TbTensor* h_out, TbTensor* act, const TbTensor* x,
                            const TbTensor* residual, const TbTensor* weight, TbTensor* q,
                            TbTensor* k, const TbTensor* gate, const TbTensor* up,
                            const TbLayerChainParams* params);

/* Register the "b200" backend (priority 200, TB_DEVICE_CUDA).  Its ops take
 * device tensors only: a host tensor gets TB_ERR_INVALID_ARG (no CPU
 * fallback inside the backend).  Idempotent. */
int tb_backend_b200_init(void);

/* The engine's CPU backend init (backend.h:143-148, defined in
 * src/backend/cpu/registry.c:63-84): declared here because this header
 * replaces backend.h; the engine defines it, this library does not. */
int tb_backend_cpu_init(void);

#ifdef __cplusplus
}
#endif
#endif /* TB_BACKEND_H */
