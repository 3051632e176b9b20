/*
 * tb_b200.h -- C ABI of the B200 (sm_100a) row-op library, libtb_b200.so.
 *
 * Plain pointers and sizes only.  Every data pointer below is CUDA device
 * memory unless stated otherwise; `stream` is a cudaStream_t passed as void*
 * (NULL selects the library's current stream, see tb_b200_set_stream).  All
 * kernel entry points are asynchronous on that stream and return a TbError
 * code (include/tb_types.h): TB_OK, TB_ERR_INVALID_ARG / TB_ERR_INVALID_SHAPE
 * for rejected arguments (nothing is launched), TB_ERR_UNSUPPORTED_DTYPE, or
 * TB_ERR_DEVICE when a CUDA call fails (tb_b200_last_error() has the text).
 *
 * dtype is a TbDtype value: TB_DTYPE_F32 or TB_DTYPE_BF16.  bf16 variants
 * read and write bf16 and compute in f32.
 *
 * Row layout: a [rows, cols] buffer is dense row-major (row stride = cols).
 *
 * Each kernel entry point replaces the reference's per-vector CPU kernel
 * (include/tensorbit/run/ops.h) applied once per row; the citation on each
 * declaration names the reference function whose arithmetic it reproduces.
 * The registry-level route (TbOpFn adapters behind tb_dispatch_*) is in
 * include/tb_backend.h.
 */
#ifndef TB_B200_H
#define TB_B200_H

#include "tb_types.h"

#ifdef __cplusplus
extern "C" {
#endif

#define TB_B200_ABI_VERSION 1

/* ======================================================================
 * Runtime: devices, memory, streams, status
 * (the reference has no device layer; its CUDA adapters passed host memory
 *  to kernels, src/backend/cuda/registry.c:68-78.  These are new.)
 * ====================================================================== */

/* ABI version of the loaded library (TB_B200_ABI_VERSION it was built with). */
int tb_b200_version(void);
/* Text of the last CUDA/NCCL failure seen on the calling thread ("" if none). */
const char* tb_b200_last_error(void);

/* Kernels launched by this library since it was loaded (all threads). */
unsigned long long tb_b200_launch_count(void);

int tb_b200_device_count(int* count);
int tb_b200_set_device(int device);
int tb_b200_get_device(int* device);

int tb_b200_malloc(void** ptr, size_t bytes);
int tb_b200_free(void* ptr);
/* Page-locked host memory, for fast and asynchronous host<->device copies. */
int tb_b200_malloc_host(void** ptr, size_t bytes);
int tb_b200_free_host(void* ptr);
int tb_b200_memcpy_h2d(void* dst_dev, const void* src_host, size_t bytes, void* stream);
int tb_b200_memcpy_d2h(void* dst_host, const void* src_dev, size_t bytes, void* stream);
int tb_b200_memcpy_d2d(void* dst_dev, const void* src_dev, size_t bytes, void* stream);
int tb_b200_memset(void* dst_dev, int value, size_t bytes, void* stream);

/* Current stream of the calling thread for calls given stream == NULL.
 * Initially NULL, i.e. the CUDA legacy default stream. */
int tb_b200_set_stream(void* stream);
void* tb_b200_get_stream(void);
int tb_b200_stream_sync(void* stream);
int tb_b200_sync(void);

/* Stream-ordered scratch: copy `bytes` of host memory into a new device
 * buffer allocated on `stream` (cudaMallocAsync), and release such a buffer
 * on `stream` once the work queued after it has used it. */
int tb_b200_stage_h2d(const void* src_host, size_t bytes, void** dst_dev, void* stream);
int tb_b200_stage_release(void* dev, void* stream);

/* *is_device = 1 if p is device (or managed) memory of any GPU, else 0. */
int tb_b200_is_device_ptr(const void* p, int* is_device);

/* Kernels record rejected data (for example a token id outside [0, vocab))
 * in a per-device status word instead of faulting.  This synchronises
 * `stream`, returns TB_ERR_INVALID_ARG if any flag was raised since the
 * last check (TB_OK otherwise), optionally reports the raw flags, and
 * clears them. */
int tb_b200_check_status(void* stream, unsigned int* flags_out);
#define TB_B200_FLAG_TOKEN_RANGE 0x1u   /* embedding: id < 0 or id >= vocab */
#define TB_B200_FLAG_WAIT_TIMEOUT 0x2u  /* a kernel's bounded wait gave up (its output is invalid) */
#define TB_B200_FLAG_POSITION_RANGE 0x4u /* decode attention: position outside [0, max_seq) */

/* Runs, in a one-warp kernel, the bounded mbarrier wait the staged kernels
 * use for their bulk copies.  supply != 0: one 16-byte copy completes the
 * wait, no flag.  supply == 0: the wait expects bytes no copy brings and
 * gives up after limit_us microseconds (1 .. 1000000, else
 * TB_ERR_INVALID_ARG), raising TB_B200_FLAG_WAIT_TIMEOUT; the kernel returns
 * and the context stays usable.  Read the outcome with
 * tb_b200_check_status.  No counterpart in the reference. */
int tb_b200_selftest_wait(int supply, uint32_t limit_us, void* stream);

/* ======================================================================
 * Row kernels
 * ====================================================================== */

/* Fused residual add + RMSNorm over [rows, cols]:
 *   h = x + residual                     (src/ops/residual.c:4-13)
 *   y = (h * (1/sqrtf((eps + sum h^2)/cols))) * weight   (src/ops/norm.c:4-26)
 * h_out receives h (may be NULL; may alias x or residual for an in-place
 * residual-stream update); weight may be NULL (no scaling, norm.c:20-22).
 * The normalisation uses the f32 sum, not the rounded h, in bf16 mode.  */
int tb_b200_residual_rms_norm(int dtype, int64_t rows, int64_t cols, const void* x,
                              const void* residual, const void* weight, void* h_out, void* y,
                              float eps, void* stream);

/* RMSNorm of each row (tb_cpu_rms_norm_f32, src/ops/norm.c:4-26). */
int tb_b200_rms_norm(int dtype, int64_t rows, int64_t cols, const void* x, const void* weight,
                     void* y, float eps, void* stream);

/* y = x + residual over n elements (tb_cpu_residual_add_f32, src/ops/residual.c:4-13). */
int tb_b200_residual_add(int dtype, int64_t n, const void* x, const void* residual, void* y,
                         void* stream);

/* y = x / (1 + expf(-x)) (tb_cpu_silu_f32, src/ops/activation.c:18-27). */
int tb_b200_silu(int dtype, int64_t n, const void* x, void* y, void* stream);

/* tanh-GELU (tb_cpu_gelu_f32, src/ops/activation.c:4-16). */
int tb_b200_gelu(int dtype, int64_t n, const void* x, void* y, void* stream);

/* out = silu(gate) * up, the engine's SwiGLU composition
 * (include/tensorbit/run/ops.hpp:246-248). */
int tb_b200_swiglu(int dtype, int64_t n, const void* gate, const void* up, void* out,
                   void* stream);

/* Rotary table: table[p][i] = {cosf(p*f_i), sinf(p*f_i)} for p < n_positions,
 * i < head_dim/2, f_i = 1.0f/powf(theta, (2.0f*i)/(float)head_dim), all
 * computed on the host with the C library exactly as src/ops/rope.c:52-54
 * does, then copied to table_dev (n_positions*head_dim floats). */
int tb_b200_rope_table(float theta, int head_dim, int n_positions, float* table_dev,
                       void* stream);

/* In-place interleaved-pair RoPE of q [rows, n_q_heads, head_dim] and
 * k [rows, n_kv_heads, head_dim], row r at positions[r] (device int32)
 * (tb_cpu_rope_gqa_f32, src/ops/rope.c:43-81, once per token).
 * table/table_positions: a tb_b200_rope_table for this theta and head_dim;
 * rows whose position is outside [0, table_positions), or all rows when
 * table is NULL, compute the angle's cos/sin on the device instead
 * (within 2 ulp of the C library rather than identical). */
int tb_b200_rope_rows(int dtype, int64_t rows, int n_q_heads, int n_kv_heads, int head_dim,
                      void* q, void* k, const int32_t* positions, float theta,
                      const float* table, int table_positions, void* stream);

/* Single-token RoPE at one position (the TB_OP_ROPE contract,
 * src/backend/cpu/rope.c:4-19): q [n_q_heads, head_dim], k [n_kv_heads,
 * head_dim].  cos/sin come from the host C library for that position. */
int tb_b200_rope(int dtype, int n_q_heads, int n_kv_heads, int head_dim, void* q, void* k,
                 int position, float theta, void* stream);

/* Row softmax over [rows, cols] with an optional additive mask of the same
 * shape (tb_cpu_softmax_f32, src/ops/softmax.c:4-32).  The row sum is the
 * reference's left-to-right f32 sum, reproduced exactly (not a tree sum). */
int tb_b200_softmax(int dtype, int64_t rows, int64_t cols, const void* x, const void* mask,
                    void* y, void* stream);

/* out[r] = index of the first maximum of row r; NaN never wins; a NaN at
 * index 0 keeps 0 (sample_argmax, src/main.cpp:79-89).  Bit-exact. */
int tb_b200_argmax(int dtype, int64_t rows, int64_t cols, const void* x, int32_t* out,
                   void* stream);

/* Temperature sampling of each row of f32 logits [rows, cols]: the index
 * sample_temperature (src/main.cpp:91-111) draws when its generator step
 * yields uniforms[r] (device doubles in [0, 1), one per row -- the value
 * std::generate_canonical<double, 53> makes of the std::mt19937 output that
 * std::discrete_distribution consumes).  temperature <= 0 is tb_b200_argmax
 * (uniforms unused); one column draws 0.  Rows whose weights hold a NaN draw
 * 0, as libstdc++'s lower_bound does over such a table.  The draw is the
 * reference's for the same u unless u lies within ~1e-15 of a cumulative
 * boundary where CUDA's and the C library's double exp differ by an ulp. */
int tb_b200_sample_temperature(int64_t rows, int64_t cols, const float* logits,
                               float temperature, const double* uniforms, int32_t* out,
                               void* stream);

/* INT4 / INT8 weights to f32 or bf16 on the device, bit-exact with the
 * engine's dequantisation of a .tbm layer (Model::get_weight_fp32,
 * include/tensorbit/run/model.hpp:181-225): n weights, INT4 packed two per
 * byte (element i in the low nibble of byte i / 2 when i is even, the high
 * one when odd, two's complement) or INT8 one signed byte; element i scaled
 * by scales[i / gs] (1 past n_scales), gs = group_size or n when it is 0;
 * out = (float)q * scale, rounded to nearest even for bf16.
 * src_dtype TB_DTYPE_INT4 / TB_DTYPE_INT8; out_dtype TB_DTYPE_F32 /
 * TB_DTYPE_BF16; src, scales, dst device memory. */
int tb_b200_dequant(int src_dtype, int64_t n, const void* src, const float* scales,
                    int64_t n_scales, uint32_t group_size, int out_dtype, void* dst,
                    void* stream);

/* y[out] = W[out, in] x[in] (+ bias), f32, one input vector: the engine's
 * linear layers (tb_cpu_sparse_linear_f32 / tb_cpu_dense_linear_f32,
 * src/ops/linear.c:4-53).  Sparse: one mask byte per M-group of a row
 * ([out, in / M] bytes), bit k keeps weight g*M + k; columns past
 * (in / M) * M are not used; nm_m >= 2 and nm_n < nm_m, else
 * TB_ERR_INVALID_ARG.  bias may be NULL.  Summed in a different order from
 * the reference's left-to-right chain: equal within f32 rounding. */
int tb_b200_sparse_linear(int64_t out_features, int64_t in_features, const float* x,
                          const float* w, const uint8_t* mask, const float* bias, float* y,
                          int nm_n, int nm_m, void* stream);
int tb_b200_dense_linear(int64_t out_features, int64_t in_features, const float* x,
                         const float* w, const float* bias, float* y, void* stream);

/* y[t] = table[ids[t]] for t < n_tokens; table [vocab, dim]; ids device
 * int32 (tb_cpu_embedding_f32, src/ops/embedding.c:4-14).  Bit-exact copy.
 * An id outside [0, vocab) zero-fills its row and raises
 * TB_B200_FLAG_TOKEN_RANGE (the reference reads out of bounds there). */
int tb_b200_embedding(int dtype, int64_t n_tokens, int64_t dim, int64_t vocab, const int32_t* ids,
                      const void* table, void* y, void* stream);

/* The same gather with the ids in host memory, as the engine passes them
 * (tb_dispatch_embedding, src/backend/cpu/registry.c:186-192): ids are
 * range-checked on the host (TB_ERR_INVALID_ARG, nothing queued, on any id
 * outside [0, vocab)) and staged to the device on `stream`. */
int tb_b200_embedding_host_ids(int dtype, int64_t n_tokens, int64_t dim, int64_t vocab,
                               const int32_t* ids_host, const void* table, void* y,
                               void* stream);

/* The same host-ids gather with no allocation.  For callers that cannot
 * allocate device memory where they make this call -- an engine whose
 * device memory is owned and budgeted by another allocator, or a per-token
 * decode step that must not take the synchronisation cudaMalloc implies.
 * Its scratch (the staged ids and the gather's status word) is one
 * statically sized device array inside the library, held by every GPU that
 * loads it until the process exits.  At most TB_B200_STATIC_MAX_TOKENS ids
 * per call; more returns TB_ERR_INVALID_SHAPE with nothing queued.  The
 * first call on a device looks up the array's device address once
 * (cudaGetSymbolAddress); later calls reuse it.  All calls share the array and
 * each starts by clearing the status word: calls whose work can overlap on
 * the GPU (different streams, no ordering between them) race on it.  The ids
 * are copied from ids_host on `stream`: from pageable memory the copy has
 * taken them when the call returns; from page-locked memory it reads them
 * when the stream reaches it, so the caller must not overwrite them before
 * then.  The array's device address is cached per device for the life of
 * the process; the library assumes no cudaDeviceReset while it is loaded.
 * No counterpart in the reference (its embedding is a host memcpy). */
#define TB_B200_STATIC_MAX_TOKENS 65536
int tb_b200_embedding_host_ids_static(int dtype, int64_t n_tokens, int64_t dim, int64_t vocab,
                                      const int32_t* ids_host, const void* table, void* y,
                                      void* stream);

/* One launch that runs a transformer layer's three row-op groups on their
 * own tensors: residual+RMSNorm [rows, hidden]; RoPE on q/k at per-row
 * positions; SwiGLU over [rows, intermediate] (the per-layer row ops of
 * TransformerRunner::forward, include/tensorbit/run/ops.hpp:120-248).
 * Results are identical to the three separate entry points.  A group whose
 * size is 0 (hidden, n_q_heads+n_kv_heads, or intermediate) is skipped. */
typedef struct {
    int dtype;
    int64_t rows;
    /* residual + RMSNorm */
    int64_t hidden;
    const void* x;
    const void* residual;
    const void* norm_weight;
    void* h_out;
    void* y;
    float eps;
    /* RoPE */
    int n_q_heads;
    int n_kv_heads;
    int head_dim;
    void* q;
    void* k;
    const int32_t* positions;
    float theta;
    const float* rope_table;
    int rope_table_positions;
    /* SwiGLU */
    int64_t intermediate;
    const void* gate;
    const void* up;
    void* act_out;
} TbB200LayerChain;

int tb_b200_layer_chain(const TbB200LayerChain* chain, void* stream);

/* 2:4 sparse weights in packed form: per pair of 4-column groups, one
 * float4 of the kept weights (column order within each group, 0 in an
 * unused slot) and one index byte (2 bits per slot: the kept column within
 * its group).  Half the bytes of the reference's dense-with-mask layout
 * (src/ops/linear.c:4-35), the same products summed.
 * pack: w [out, in] f32 and mask [out, in/4] bytes (bits 0..3 of a byte
 * keep columns of its group) -> vals (16-byte aligned, out * P float4s) and
 * idx (out * S bytes), P = ceil((in/4) / 2), S = P rounded up to a multiple
 * of 128; within a row the byte of pair p = 128 s + 32 u + l (l < 32,
 * u < 4) is at 128 s + 4 l + u, so a lane loads its four bytes of a
 * 128-pair step as one 32-bit word.  A group with more than two
 * mask bits set sets *unpackable_dev to 1 (the layer must stay dense-with-
 * mask); the caller zeroes it first and reads it after the stream.
 * linear: y = W x (+ bias) from the packed form; (in/4) must be even, x and
 * vals 16-byte aligned; bias may alias y. */
int tb_b200_sparse24_pack(int64_t out_features, int64_t in_features, const float* w,
                          const uint8_t* mask, void* vals, uint8_t* idx, int* unpackable_dev,
                          void* stream);
int tb_b200_sparse24_linear(int64_t out_features, int64_t in_features, const float* x,
                            const void* vals, const uint8_t* idx, const float* bias, float* y,
                            void* stream);

/* ======================================================================
 * Decoder forward on the device (TransformerRunner)
 * ====================================================================== */

/* Attention row layouts of tb_b200_decode_attention / the runner. */
#define TB_B200_ATTN_REFERENCE 0 /* the rows the reference's runner passes on */
#define TB_B200_ATTN_STANDARD 1  /* query row `position` of every head */

/* Single-token attention over one layer's KV cache (the attention step of
 * TransformerRunner::forward, include/tensorbit/run/ops.hpp:162-204, over
 * tb_cpu_scaled_dot_product_f32, src/ops/attention.c:5-69), f32.
 *   position  device int32: the token's position p, in [0, max_seq);
 *   q [n_heads * head_dim], k/v [n_kv_heads * head_dim]: the token's
 *             projections after RoPE; k and v are also written to cache row p;
 *   k_cache/v_cache [max_seq, n_kv_heads * head_dim]: rows 0 .. p-1 hold the
 *             earlier tokens';
 *   out [n_heads * head_dim].
 * Scale 1/sqrtf(head_dim).  TB_B200_ATTN_REFERENCE: out holds the first
 * n_heads * head_dim floats of the reference's [n_heads, p+1, head_dim]
 * causal attention over q repeated p+1 times -- row r is head r / (p+1)
 * attending keys 0 .. r % (p+1).  TB_B200_ATTN_STANDARD: row h is head h
 * attending keys 0 .. p.  Query head h reads k/v head h / (n_heads /
 * n_kv_heads).  head_dim <= 256; a position outside [0, max_seq) writes
 * nothing and raises TB_B200_FLAG_POSITION_RANGE. */
int tb_b200_decode_attention(int mode, int n_heads, int n_kv_heads, int head_dim, int max_seq,
                             const int32_t* position, const float* q, const float* k,
                             const float* v, float* k_cache, float* v_cache, float* out,
                             void* stream);

/* One weight tensor of a model, as the reference's Model hands it out
 * (Model::get_weights / get_mask / get_scales, include/tensorbit/run/
 * model.hpp:154-177).  data: [rows, cols] in host or device memory (the
 * runner copies host data to the device); NULL means the tensor is absent.
 * dtype TB_DTYPE_F32, TB_DTYPE_INT8 or TB_DTYPE_INT4 (dequantised once to
 * f32 on the device, as Model::get_weight_fp32 does per use, model.hpp:
 * 181-225).  mask: rows * (cols / 4) bytes of 2:4 groups, NULL for a dense
 * projection. */
typedef struct {
    const void* data;
    int dtype;
    int64_t rows;
    int64_t cols;
    const uint8_t* mask;
    const float* scales;
    int64_t n_scales;
    uint32_t group_size;
} TbB200Weight;

/* One decoder layer: the tensors ops.hpp:97-105 looks up.  A layer without
 * q, k or v is skipped (ops.hpp:109); without o, no attention output
 * projection; without gate or up, no MLP; without down, no MLP residual.
 * Norm weights: [hidden] f32, NULL for none. */
typedef struct {
    TbB200Weight q, k, v, o, gate, up, down;
    const float* input_norm;
    const float* post_norm;
} TbB200RunnerLayer;

/* A model for the device runner: TransformerRunner's normalised config
 * (ops.hpp:291-323, every field given) and its tensors. */
typedef struct {
    int hidden, n_heads, n_kv_heads, head_dim, intermediate, vocab, max_seq, layers;
    float norm_eps;
    float rope_theta;
    int attention;                  /* TB_B200_ATTN_REFERENCE or _STANDARD */
    int use_graph;                  /* nonzero: replay each token as one CUDA graph */
    TbB200Weight embed;             /* [vocab, hidden] */
    const float* final_norm;        /* [hidden] or NULL */
    TbB200Weight lm_head;           /* [vocab, hidden]; data NULL: the embedding table */
    const TbB200RunnerLayer* layer; /* [layers] */
} TbB200RunnerDesc;

/* TransformerRunner on the device (include/tensorbit/run/ops.hpp:33-288):
 * weights, activations and the KV cache live in HBM; each forward runs the
 * token's whole decoder step on the runner's own stream.  The norms cover
 * `hidden` floats (the reference normalises its max(hidden, vocab) state
 * vector, reading past the hidden-sized norm weights when vocab > hidden).
 * create: uploads / dequantises what is not already f32 on the device
 * (borrowed device tensors must outlive the runner), packs every masked
 * projection whose groups keep at most two weights (tb_b200_sparse24_pack;
 * an uploaded dense copy is freed after packing), allocates the cache and
 * builds the RoPE table with the host C library. */
int tb_b200_runner_create(const TbB200RunnerDesc* desc, void** runner);
/* Run one token at the next position; *logits_dev (optional) receives the
 * runner's device logits [vocab], valid until the next forward.  A token
 * outside [0, vocab) returns TB_ERR_INVALID_ARG and a full cache (max_seq
 * positions used) TB_ERR_INVALID_SHAPE, both with nothing queued.
 * Asynchronous: the runner's stream orders later calls. */
int tb_b200_runner_forward(void* runner, int32_t token, const float** logits_dev);
/* Copy the last logits to host memory (synchronises the runner's stream). */
int tb_b200_runner_logits(void* runner, float* logits_host);
/* Start a new sequence at position 0 (TransformerRunner::reset, ops.hpp:52). */
int tb_b200_runner_reset(void* runner);
int tb_b200_runner_position(void* runner, int* position);
/* The runner's stream (cudaStream_t), for callers that order work after it. */
int tb_b200_runner_stream(void* runner, void** stream);
/* Kernels one forward launches (the graph's nodes when use_graph is set). */
int tb_b200_runner_launches_per_token(void* runner, int* launches);
int tb_b200_runner_destroy(void* runner);

/* ======================================================================
 * .tbm model containers read into device memory
 * ====================================================================== */

/* The model config of a .tbm index, the reference's TbModelConfig
 * (include/tensorbit/run/model.h:34-46), read as its parser reads it
 * (src/model.c:280-475): a "config" object clears the whole config (an
 * "architecture" read before it included), defaults norm_eps to 1e-6 and
 * rope_theta to 10000, sets num_kv_heads = num_heads when 0 and head_dim =
 * hidden_size / num_heads; without one every field is 0. */
typedef struct {
    char architecture[64];
    int hidden_size, num_heads, num_kv_heads, intermediate_size, vocab_size, max_seq_len,
        num_layers;
    float norm_eps, rope_theta;
    int head_dim;
} TbB200TbmConfig;

/* One tensor of a loaded container: its index entry (the reference's
 * TbLayerDesc, include/tensorbit/run/model.h:15-26) and DEVICE pointers to
 * its bytes, copied unchanged from the file: weights (weight_bytes: INT4
 * ceil(n/2), INT8 n, else n elements), mask (num_mask_bytes; NULL when 0)
 * and f32 scales (scale_count of them, quantized tensors only; else NULL).
 * The pointers stay valid until tb_b200_tbm_free. */
typedef struct {
    char name[128];
    int64_t shape[2];
    int dtype;
    uint32_t nm_n, nm_m;
    int64_t num_weights, num_mask_bytes, scale_count;
    uint32_t group_size;
    const void* weights;
    const uint8_t* mask;
    const float* scales;
    int64_t weight_bytes;
} TbB200TbmTensor;

/* Read a .tbm container (docs/TBM_FORMAT.md) into one device allocation on
 * the current device: the file is mapped read-only, its JSON index parsed as
 * tb_model_load_tbm parses it (src/model.c:482-580), and every tensor's
 * weights, mask bytes and scales -- located as the reference's zero-copy
 * views locate them (src/model.c:681-739) -- streamed to the device through
 * page-locked staging buffers on `stream`; returns once they have landed.
 * Errors: TB_ERR_FILE_OPEN / TB_ERR_FILE_READ, TB_ERR_TRUNCATED (a file
 * shorter than 20 bytes, a bad index length, or a tensor running past the
 * end of the file), TB_ERR_JSON_PARSE, TB_ERR_DEVICE.  A tensor whose .tb
 * header has a bad magic gets no device bytes; tb_b200_tbm_tensor reports it
 * as TB_ERR_BAD_MAGIC, as the reference's views do. */
int tb_b200_tbm_load(const char* path, void* stream, void** model);
int tb_b200_tbm_config(const void* model, TbB200TbmConfig* cfg);
int tb_b200_tbm_count(const void* model, int* count);
/* Index of the tensor named `name` (tb_model_find_layer), or
 * TB_ERR_LAYER_NOT_FOUND. */
int tb_b200_tbm_find(const void* model, const char* name, int* index);
int tb_b200_tbm_tensor(const void* model, int index, TbB200TbmTensor* out);
/* A device-runner description of the loaded model, as TransformerRunner
 * finds its tensors (include/tensorbit/run/ops.hpp:61-116, 259-276:
 * llama, gpt-j and bare names; the lm head falls back to the embedding) with
 * its normalised config (ops.hpp:291-323).  `layers` receives the per-layer
 * descriptions (capacity max_layers); the weights are borrowed from the
 * loaded model, which must outlive any runner made from it.  Norm weights
 * must be f32 (TB_ERR_UNSUPPORTED_DTYPE otherwise). */
int tb_b200_tbm_runner_desc(const void* model, int attention, int use_graph,
                            TbB200RunnerDesc* desc, TbB200RunnerLayer* layers, int max_layers);
int tb_b200_tbm_free(void* model);

/* ======================================================================
 * Multi-GPU (one process per GPU)
 * ====================================================================== */

/* Contiguous split of `total` items over `parts`: part p gets
 * [lo, hi); the first total%parts parts get one extra item. */
int tb_b200_partition(int64_t total, int parts, int part, int64_t* lo, int64_t* hi);

/* The exchange plan of tb_b200_embedding_sharded for `rank` (host only,
 * no device work): with ids (n_tokens host int32, all in [0, vocab)),
 *   send_counts[d]  rows this rank sends to rank d (0 for d == rank);
 *   send_rows       this rank's table-shard rows to send, destination-major,
 *                   token order within a destination (capacity n_tokens);
 *   recv_counts[s]  rows this rank receives from rank s;
 *   recv_rows       output rows (within this rank's token part) the received
 *                   rows go to, source-major, token order (capacity n_tokens);
 *   local_dst/src   (output row, table-shard row) of tokens this rank owns
 *                   both ends of; *n_local of them (capacity n_tokens). */
int tb_b200_shard_plan(int64_t n_tokens, int64_t vocab, int nranks, int rank,
                       const int32_t* ids_host, int64_t* send_counts, int64_t* recv_counts,
                       int32_t* send_rows, int32_t* recv_rows, int32_t* local_dst,
                       int32_t* local_src, int64_t* n_local);

/* NCCL communicator of this process.  Rank 0 calls tb_b200_comm_unique_id
 * and shares the 128 bytes with the other ranks out of band; every rank
 * then calls tb_b200_comm_init with its own rank on its own device. */
#define TB_B200_COMM_ID_BYTES 128
int tb_b200_comm_unique_id(void* id_out);
int tb_b200_comm_init(int nranks, int rank, const void* unique_id, int device);
int tb_b200_comm_destroy(void);
int tb_b200_comm_info(int* rank, int* nranks);

/* Bounded wait for the work queued on `stream` so far -- the exchanges of
 * tb_b200_embedding_sharded among it.  Polls the stream and the
 * communicator's error state every few microseconds.  TB_OK once the work
 * is done.  If the communicator reports an error, or the work is not done
 * after TB_B200_COMM_TIMEOUT_S seconds (environment, default 120; a peer
 * that never posts its side of an exchange), the communicator is aborted
 * (its kernels still waiting for peers end, with their output invalid),
 * released, and TB_ERR_DEVICE is returned; tb_b200_comm_init may then make
 * a new one.  The reference has no communication layer: no counterpart. */
int tb_b200_comm_wait(void* stream);

/* Vocab-sharded embedding gather over the communicator.  Every rank holds
 * the same n_tokens ids (host int32), the table rows of its vocab part
 * (tb_b200_partition(vocab, nranks, rank)) in table_shard, and receives the
 * rows of its token part (tb_b200_partition(n_tokens, nranks, rank)) in
 * y_local.  Owned rows are copied locally; the rest arrive from their
 * owners through one grouped NCCL send/recv exchange.  Bit-exact with
 * tb_cpu_embedding_f32 over the full table.  Ids outside [0, vocab) return
 * TB_ERR_INVALID_ARG before any work is queued.  Returns once the exchange
 * is queued on `stream` (that host-side enqueue is bounded by
 * TB_B200_COMM_TIMEOUT_S); the exchange runs asynchronously, and
 * tb_b200_comm_wait bounds the wait for it. */
int tb_b200_embedding_sharded(int dtype, int64_t n_tokens, int64_t dim, int64_t vocab,
                              const int32_t* ids_host, const void* table_shard, void* y_local,
                              void* stream);

/* Symmetric memory of the communicator (NCCL windows): every rank calls
 * tb_b200_comm_window_alloc with the same size, in the same order, and gets
 * `bytes` (rounded up to 4 KB) of device memory that NCCL maps into every
 * other rank's address space; tb_b200_comm_window_free (collective, same
 * order) releases it, and tb_b200_comm_destroy releases what is left.
 * TB_ERR_DEVICE when the loaded NCCL has no windows.  Bounded like every
 * host-side wait on the communicator.  No counterpart in the reference. */
int tb_b200_comm_window_alloc(size_t bytes, void** ptr);
int tb_b200_comm_window_free(void* ptr);

/* The vocab-sharded gather as one kernel over the communicator's symmetric
 * memory: the same computation as tb_b200_embedding_sharded (the
 * reference's per-token row copy, src/ops/embedding.c:4-14, over a table
 * split by vocabulary rows), with no exchange step.  Every rank keeps its
 * table part (tb_b200_partition(vocab, nranks, rank)) at the same byte
 * offset of a window from tb_b200_comm_window_alloc and passes its own
 * pointer as `shard`; ids (n_tokens DEVICE int32) are the tokens whose rows
 * this call writes to y [n_tokens, dim] -- usually this rank's token part.
 * Each row is read from its owner's window (a peer load over NVLink when the
 * owner is another GPU; nothing waits on another GPU, the shards being
 * written before any gather) and written once: bit-exact with
 * tb_cpu_embedding_f32 over the full table.  Ids outside [0, vocab) give a
 * zero row and raise TB_B200_FLAG_TOKEN_RANGE. */
int tb_b200_embedding_sharded_window(int dtype, int64_t n_tokens, int64_t dim, int64_t vocab,
                                     const int32_t* ids, const void* shard, void* y,
                                     void* stream);

/* Peer memory of the other GPUs of one box, through CUDA IPC, for the
 * one-kernel sharded gather below.  The owner of a device buffer exports a
 * handle (TB_B200_P2P_HANDLE_BYTES bytes) and the buffer's offset within its
 * allocation; the handle and offset go to the other processes out of band;
 * each opens them into a device pointer valid in its own context until it
 * closes it (tb_b200_p2p_close, with the same offset).  The owner must keep
 * the buffer alive until every importer has closed it. */
#define TB_B200_P2P_HANDLE_BYTES 64
int tb_b200_p2p_export(const void* dev_ptr, void* handle_out, int64_t* offset_out);
int tb_b200_p2p_import(const void* handle, int64_t offset, void** dev_ptr_out);
int tb_b200_p2p_close(void* dev_ptr, int64_t offset);

/* Vocab-sharded embedding gather as one kernel, no collective.  The same
 * computation as tb_b200_embedding_sharded (the reference's per-token row
 * copy, src/ops/embedding.c:4-14, over a table split by vocabulary rows):
 * shards[r] (rank order, nranks <= 8) is rank r's table part
 * (tb_b200_partition(vocab, nranks, r)) -- this rank's own pointer for its
 * own part, imported pointers for the others' -- and ids (n_tokens DEVICE
 * int32) are the tokens whose rows this call writes to y [n_tokens, dim].
 * Each row is read from its owner's memory (a peer load over NVLink when
 * the owner is another GPU) and written once: bit-exact with
 * tb_cpu_embedding_f32 over the full table.  Ids outside [0, vocab) give a
 * zero row and raise TB_B200_FLAG_TOKEN_RANGE (tb_b200_check_status). */
int tb_b200_embedding_sharded_p2p(int dtype, int64_t n_tokens, int64_t dim, int64_t vocab,
                                  const int32_t* ids, const void* const* shards, int nranks,
                                  void* y, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* TB_B200_H */
