// runner_kernels.h -- the fused kernels of the device decoder step
// (k_runner.cu, k_attention.cu) as runner.cu launches them.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace tbh {

struct GemvSeg {
    const void* w;       // dense f32 [rows, cols], the packed float4 values, or INT8/INT4 bytes
    const uint8_t* idx;  // packed index bytes (packed layout only)
    float* y;            // output [rows]
    int64_t rows;
    const float* scales; // INT8/INT4: one scale per group, every group present
    int64_t n_scales;
    int gshift;          // INT8/INT4: log2(group size), 31 for one group
};

enum GemvLayout { kDense = 0, kPacked = 1, kInt8 = 2, kInt4 = 3 };
enum GemvEpi { kPlain = 0, kResidual = 1, kRope = 2, kSwiglu = 3 };

struct GemvArgs {
    GemvSeg seg[3];
    int nseg;
    int64_t cols;        // input features
    const float* x;      // input vector [cols]
    const float* res;    // kResidual: y = res + W x (res may be y)
    float* act;          // kSwiglu: output [rows]
    const float2* rope;  // kRope: (cos, sin) table [rope_positions, head_dim / 2]
    int rope_positions;
    const int32_t* pos;  // kRope: device position
    int head_dim;
    int rope_segs;       // segments 0 .. rope_segs-1 are rotated
    int32_t* advance;    // non-null: *advance += 1 once the kernel has run
    unsigned* status;
    int norm;            // nonzero: the GEMV reads rms_norm(x) * norm_w instead of x
    const float* norm_w; // norm weight [cols] or NULL
    float eps;
    float* norm_out;     // non-null: CTA 0 also stores the normalised x there
    int64_t units;       // set by fused_gemv: row pairs (or gate/up rows)
    int ks;              // set by fused_gemv: warps sharing one unit
};

// One fused GEMV launch over 1-3 segments sharing x (programmatic dependent
// launch).  layout kDense needs cols % 4 == 0, kPacked cols % 8 == 0, kInt8 and
// kInt4 cols % 32 == 0 and a group size of at least 8 (a power of two); x and
// the weights 16-byte aligned.  kSwiglu takes two segments of equal rows.
// With norm set, every CTA normalises x into shared memory first (cols * 4
// bytes; fused_gemv_setup opts in to more than 48 KB).
int fused_gemv(const GemvArgs& a, int layout, int epi, cudaStream_t s);
int fused_gemv_setup(int64_t cols);
// RMSNorm of one f32 vector, one CTA, programmatic dependent launch.
int runner_norm(int64_t n, const float* x, const float* w, float* y, float eps, cudaStream_t s);
// Opt the attention kernels in to the shared memory max_seq keys need.
int decode_attention_setup(int head_dim, int max_seq);
// splits > 1: rows of more than 512 keys are split over that many CTAs,
// which leave (max, sum, weighted v) in part (n_heads * splits * (head_dim
// + 2) floats) and count themselves in counters (n_heads ints, zero before
// the first launch; the last CTA of a row resets its counter).
int decode_attention_launch(int mode, int n_heads, int n_kv_heads, int head_dim, int max_seq,
                            const int32_t* position, const float* q, const float* k,
                            const float* v, float* k_cache, float* v_cache, float* out,
                            cudaStream_t s, bool pdl, int splits, float* part, int* counters);
int decode_attention_splits(int n_rows, int max_seq);

}  // namespace tbh
