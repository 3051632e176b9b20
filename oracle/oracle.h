/*
 * oracle.h -- CPU oracle for the tensorbit-run row-op hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library links, loads or
 * calls this code; it exists so the parity tests, the smoke check and the
 * CPU-baseline leg of bench.py have an independent CPU answer to compare the
 * sm_100a kernels against.
 *
 * Two implementations sit behind the same row-batched driver API:
 *   ORC_IMPL_PORT  -- port.c, a restatement of the reference's per-vector C
 *                     kernels (each function cites the file:line it follows),
 *                     compiled with the reference's own Release/SIMD flags
 *                     (-O3 -mavx2 -mfma, gnu11) so FMA contraction matches;
 *   ORC_IMPL_REF   -- the reference's own src/ops/*.c, compiled unmodified
 *                     from the reference tree into oracle/_ref/libtbref.so by
 *                     oracle/Makefile and resolved at run time with dlopen.
 * The port is pinned to the reference by tests/test_oracle.py (bit-exact on
 * seeded inputs) and by the committed golden checksums in tests/golden/.
 *
 * Row semantics (both implementations): a [rows, cols] row-major buffer is
 * processed by calling the reference's per-vector kernel once per row.
 */
#ifndef TB_ORACLE_H
#define TB_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_IMPL_PORT = 0, ORC_IMPL_REF = 1 };
/* dtype codes follow TbDtype (include/tensorbit/run/common.h:89-99). */
enum { ORC_F32 = 0, ORC_BF16 = 2 };

/* ---- per-vector restatements (port.c) ---------------------------------- */
int orc_rms_norm_f32(size_t n, const float* x, const float* weight, float* y, float eps);
int orc_residual_add_f32(size_t n, const float* x, const float* residual, float* y);
int orc_gelu_f32(size_t n, const float* x, float* y);
int orc_silu_f32(size_t n, const float* x, float* y);
int orc_rope_gqa_f32(int n_q_heads, int n_kv_heads, int head_dim, float* q, float* k,
                     int position, float theta_base);
int orc_softmax_f32(size_t n, const float* x, const float* mask, float* y);
int orc_embedding_f32(const int* token_ids, int n_tokens, int embedding_dim, const float* table,
                      float* y);
int orc_argmax_f32(const float* logits, int n);
int orc_swiglu_f32(size_t n, const float* gate, const float* up, float* out);
int orc_sparse_linear_f32(size_t out_features, size_t in_features, const float* x, const float* w,
                          const uint8_t* mask, const float* bias, float* y, int nm_n, int nm_m);
int orc_dense_linear_f32(size_t out_features, size_t in_features, const float* x, const float* w,
                         const float* bias, float* y);

/* bf16 <-> f32 (round to nearest even; NaN stays a quiet NaN). */
uint16_t orc_f32_to_bf16(float f);
float orc_bf16_to_f32(uint16_t h);

/* ---- reference library ------------------------------------------------- */
/* Load oracle/_ref/libtbref.so (the reference's own kernels).  0 on success. */
int orc_load_ref(const char* path);
int orc_ref_loaded(void);

/* ---- row-batched drivers (rows.c) --------------------------------------
 * impl: ORC_IMPL_PORT / ORC_IMPL_REF.  dtype: ORC_F32 / ORC_BF16 (bf16 rows
 * are widened to f32, computed by the f32 kernel, rounded back RNE).
 * nthreads <= 1 runs on the calling thread; more splits rows into contiguous
 * blocks, one pthread each.  Return 0, or a nonzero TbError-style code.   */
int orc_rows_residual_rms_norm(int impl, int dtype, int64_t rows, int64_t cols, const void* x,
                               const void* residual, const void* weight, void* h_out, void* y,
                               float eps, int nthreads);
int orc_rows_rms_norm(int impl, int dtype, int64_t rows, int64_t cols, const void* x,
                      const void* weight, void* y, float eps, int nthreads);
int orc_rows_residual_add(int impl, int dtype, int64_t rows, int64_t cols, const void* x,
                          const void* residual, void* y, int nthreads);
int orc_rows_gelu(int impl, int dtype, int64_t rows, int64_t cols, const void* x, void* y,
                  int nthreads);
int orc_rows_silu(int impl, int dtype, int64_t rows, int64_t cols, const void* x, void* y,
                  int nthreads);
int orc_rows_swiglu(int impl, int dtype, int64_t rows, int64_t cols, const void* gate,
                    const void* up, void* out, int nthreads);
int orc_rows_rope(int impl, int dtype, int64_t rows, int n_q_heads, int n_kv_heads, int head_dim,
                  void* q, void* k, const int32_t* positions, float theta, int nthreads);
int orc_rows_softmax(int impl, int dtype, int64_t rows, int64_t cols, const void* x,
                     const void* mask, void* y, int nthreads);
int orc_rows_argmax(int impl, int dtype, int64_t rows, int64_t cols, const void* x, int32_t* out,
                    int nthreads);
int orc_rows_embedding(int impl, int dtype, int64_t n_tokens, int64_t dim, const int32_t* ids,
                       const void* table, void* y, int nthreads);

/* ---- temperature sampling (sampling.c) --------------------------------
 * The reference's sample_temperature (src/main.cpp:91-111) with the draw of
 * libstdc++'s discrete_distribution restated for a given uniform u (the
 * generate_canonical<double, 53> value of its mt19937 step).              */
typedef struct {
    uint32_t s[624];
    int i;
} orc_mt;
void orc_mt_seed(orc_mt* st, uint32_t seed);
uint32_t orc_mt_next(orc_mt* st);
double orc_canonical53(orc_mt* st);
/* count successive canonical doubles of mt19937(seed), two outputs each. */
void orc_uniforms(uint32_t seed, int64_t count, double* out);
/* scratch: n doubles.  Returns the drawn index (-1 without scratch). */
int orc_sample_temperature_u(const float* logits, int n, float temperature, double u,
                             double* scratch);
/* Row driver: logits f32 [rows, cols], u [rows] -> out [rows]. */
int orc_rows_sample_temperature(int64_t rows, int64_t cols, const float* logits,
                                float temperature, const double* u, int32_t* out, int nthreads);

/* ---- INT4 / INT8 weight dequantisation (dequant.c) --------------------
 * Model::get_weight_fp32 (include/tensorbit/run/model.hpp:181-225):
 * dtype 7 = INT8, 8 = INT4 (TbDtype).                                     */
int orc_dequant_f32(int dtype, size_t n, const void* src, const float* scales, size_t n_scales,
                    uint32_t group_size, float* dst);

/* ---- single-token decoder forward (runner.c) ---------------------------
 * TransformerRunner::forward (include/tensorbit/run/ops.hpp:79-288) over f32
 * weights.  A projection with a mask runs as 2:4 groups, without one dense.
 * Norm weights may be NULL (no scaling); lm_head NULL uses the embedding
 * table (tied weights).  logits: [n_tokens, vocab], the logits after each
 * token, positions 0 .. n_tokens-1 from a fresh state.                    */
enum { ORC_ATTN_REFERENCE = 0, ORC_ATTN_STANDARD = 1 };
typedef struct {
    const float* w;      /* [rows, cols] f32, NULL: absent */
    const uint8_t* mask; /* rows * (cols / 4) bytes, NULL: dense */
    int64_t rows, cols;
} orc_lin;
typedef struct {
    orc_lin q, k, v, o, gate, up, down;
    const float* in_norm;
    const float* post_norm;
} orc_layer;
typedef struct {
    const float* embed;      /* [vocab, hidden] */
    const float* final_norm; /* [hidden] or NULL */
    const float* lm_head;    /* [vocab, hidden] or NULL */
    const orc_layer* layers; /* [layers] */
} orc_model;
typedef struct {
    int hidden, n_heads, n_kv_heads, head_dim, intermediate, vocab, max_seq, layers;
    float norm_eps, rope_theta;
    int attention; /* ORC_ATTN_REFERENCE / ORC_ATTN_STANDARD */
} orc_runner_cfg;
int orc_runner_run(const orc_runner_cfg* cfg, const orc_model* model, int n_tokens,
                   const int32_t* tokens, float* logits);

#ifdef __cplusplus
}
#endif
#endif /* TB_ORACLE_H */
