// tb_internal.h -- host-side plumbing shared by the library's .cu files:
// stream resolution, CUDA error capture, per-device state.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/tb_b200.h"

namespace tbh {

// Record `err` (with `what`) as the calling thread's last error text.
void set_error(const char* what, cudaError_t err);
void set_error_text(const char* text);

// Stream to launch on: `s` if given, else the thread's current stream.
cudaStream_t stream_of(void* s);

// Per-device state, created on first use on the current device.
struct DeviceState {
    int device = -1;
    unsigned int* status = nullptr;  // device word of TB_B200_FLAG_* bits
    int sm_count = 0;
    size_t smem_optin = 0;
};
// State of the current device, or nullptr (error already recorded).
DeviceState* current_device_state();

bool aligned16(const void* p);

// Grid size for a grid-stride elementwise kernel: enough CTAs to keep every
// SM busy, never more than there is work for.
int ew_grid(int64_t work_items, int threads, const DeviceState* ds, int ctas_per_sm = 8);

// f_i = 1.0f/powf(theta, (2.0f*i)/(float)head_dim) for i < head_dim/2,
// with the host C library (src/ops/rope.c:52).
void rope_inv_freq(float theta, int head_dim, float* out);

// Thread layout of the RMSNorm bodies for rows of `nvec` vectors: G threads
// per row (a power of two, 32..max_group), `items` vectors per thread (at
// most 4; 0 means the row is too wide for registers), CTA size `threads`.
struct NormCfg {
    int G, items, threads;
};
inline NormCfg norm_cfg(int64_t nvec, int max_group) {
    NormCfg c;
    if (nvec <= 32 * 4) {
        c.G = 32;
        c.items = (int)((nvec + 31) / 32);
    } else {
        int g = 1;
        while (g < (nvec + 3) / 4) g <<= 1;
        c.G = g > max_group ? max_group : g;
        const int64_t it = (nvec + c.G - 1) / c.G;
        c.items = it > 4 ? 0 : (int)it;  // wider rows: the two-pass kernel
    }
    if (c.items > 2) c.items = 4;
    c.threads = c.G < 256 ? 256 : c.G;
    return c;
}

// f32 softmax staged through shared memory (k_softmax_staged.cu): TB_OK
// after launching, 1 when the shape is not one it handles, else an error.
int softmax_staged_f32(int64_t rows, int64_t cols, const float* x, float* y, cudaStream_t s);
// f32 softmax with each row split over a thread-block cluster
// (k_softmax_cluster.cu): same return convention.
int softmax_cluster_f32(int64_t rows, int64_t cols, const float* x, float* y, cudaStream_t s);
// Whether f32 softmax tries the cluster kernel first: TB_B200_SOFTMAX=cluster
// in the environment (read at each call); otherwise the staged and tiled
// kernels.
bool softmax_use_cluster();

}  // namespace tbh

#define TB_CUDA_TRY(call)                                       \
    do {                                                        \
        cudaError_t tb_e_ = (call);                             \
        if (tb_e_ != cudaSuccess) {                             \
            tbh::set_error(#call, tb_e_);                       \
            return TB_ERR_DEVICE;                               \
        }                                                       \
    } while (0)

namespace tbh {
// Number of kernels this library has launched (host-side count).
void count_launch();
}  // namespace tbh

// After a <<<>>> launch: count it and report a launch-configuration failure.
#define TB_LAUNCH_CHECK(name)                                   \
    do {                                                        \
        tbh::count_launch();                                    \
        cudaError_t tb_e_ = cudaGetLastError();                 \
        if (tb_e_ != cudaSuccess) {                             \
            tbh::set_error(name, tb_e_);                        \
            return TB_ERR_DEVICE;                               \
        }                                                       \
    } while (0)
