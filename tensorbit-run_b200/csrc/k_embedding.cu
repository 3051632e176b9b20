// k_embedding.cu -- token-embedding gather, a bit-exact row copy.
//
// Reference (tb_cpu_embedding_f32, src/ops/embedding.c:4-14):
//   y[t] = table[ids[t]]   (memcpy of one row per token, no range check).
// The copy is dtype-agnostic: rows move as raw bytes, 16 at a time when the
// row size and both pointers allow it.  An id outside [0, vocab) -- memory
// the reference would read out of bounds -- zero-fills its output row and
// raises TB_B200_FLAG_TOKEN_RANGE in the device status word.
//
// Data path: HBM bound, 2*R*H*s bytes (+4R for the ids).  One CTA per
// token for wide rows, several tokens per CTA (a warp each) for short rows;
// UNROLL 16-byte chunks in flight per thread.
#include <mutex>

#include "tb_device.cuh"
#include "tb_internal.h"

namespace {

template <typename W, int UNROLL>
__device__ __forceinline__ void copy_row(const W* __restrict__ src, W* __restrict__ dst,
                                         int64_t n, int first, int step, bool zero) {
    int64_t i = first;
    for (; i + (UNROLL - 1) * (int64_t)step < n; i += UNROLL * (int64_t)step) {
        W v[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) v[u] = zero ? W{} : src[i + u * step];
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) dst[i + u * step] = v[u];
    }
    for (; i < n; i += step) dst[i] = zero ? W{} : src[i];
}

// Rows of `words` W-sized words; `group` threads per token.
template <typename W>
__global__ void __launch_bounds__(256)
k_embed(const int32_t* __restrict__ ids, const W* __restrict__ table, W* __restrict__ y,
        int64_t n_tokens, int64_t words, int64_t vocab, int group, unsigned int* status) {
    const int64_t t = (int64_t)blockIdx.x * (blockDim.x / group) + threadIdx.x / group;
    if (t >= n_tokens) return;
    const int lane = threadIdx.x % group;
    const int32_t id = ids[t];
    const bool bad = id < 0 || (int64_t)id >= vocab;
    if (bad && lane == 0) atomicOr(status, tbk::kFlagTokenRange);
    copy_row<W, 4>(table + (bad ? 0 : (int64_t)id * words), y + t * words, words, lane, group,
                   bad);
}

template <typename W>
int launch(int64_t n_tokens, int64_t row_bytes, int64_t vocab, const int32_t* ids,
           const void* table, void* y, unsigned int* status, cudaStream_t s) {
    const int64_t words = row_bytes / (int64_t)sizeof(W);
    int group = 32;
    while (group < 256 && group * 4 < words) group <<= 1;
    const int per_cta = 256 / group;
    const unsigned grid = (unsigned)((n_tokens + per_cta - 1) / per_cta);
    k_embed<W><<<grid, 256, 0, s>>>(ids, static_cast<const W*>(table), static_cast<W*>(y),
                                    n_tokens, words, vocab, group, status);
    TB_LAUNCH_CHECK("embedding kernel");
    return TB_OK;
}

}  // namespace

extern "C" int tb_b200_embedding(int dtype, int64_t n_tokens, int64_t dim, int64_t vocab,
                                 const int32_t* ids, const void* table, void* y, void* stream) {
    if (n_tokens < 0 || dim < 0 || vocab < 0 || n_tokens > INT32_MAX) return TB_ERR_INVALID_SHAPE;
    if (dtype != TB_DTYPE_F32 && dtype != TB_DTYPE_BF16) return TB_ERR_UNSUPPORTED_DTYPE;
    if (n_tokens == 0 || dim == 0) return TB_OK;
    if (!ids || !table || !y) return TB_ERR_INVALID_ARG;
    tbh::DeviceState* ds = tbh::current_device_state();
    if (!ds) return TB_ERR_DEVICE;
    cudaStream_t s = tbh::stream_of(stream);
    const int64_t row_bytes = dim * (dtype == TB_DTYPE_F32 ? 4 : 2);
    const uintptr_t a = reinterpret_cast<uintptr_t>(table) | reinterpret_cast<uintptr_t>(y);
    if (row_bytes % 16 == 0 && (a & 15) == 0)
        return launch<uint4>(n_tokens, row_bytes, vocab, ids, table, y, ds->status, s);
    if (row_bytes % 4 == 0 && (a & 3) == 0)
        return launch<uint32_t>(n_tokens, row_bytes, vocab, ids, table, y, ds->status, s);
    return launch<uint16_t>(n_tokens, row_bytes, vocab, ids, table, y, ds->status, s);
}

extern "C" int tb_b200_embedding_host_ids(int dtype, int64_t n_tokens, int64_t dim, int64_t vocab,
                                          const int32_t* ids_host, const void* table, void* y,
                                          void* stream) {
    if (n_tokens < 0 || dim < 0 || vocab < 0 || n_tokens > INT32_MAX) return TB_ERR_INVALID_SHAPE;
    if (dtype != TB_DTYPE_F32 && dtype != TB_DTYPE_BF16) return TB_ERR_UNSUPPORTED_DTYPE;
    if (n_tokens == 0 || dim == 0) return TB_OK;
    if (!ids_host || !table || !y) return TB_ERR_INVALID_ARG;
    for (int64_t t = 0; t < n_tokens; ++t)
        if (ids_host[t] < 0 || (int64_t)ids_host[t] >= vocab) return TB_ERR_INVALID_ARG;
    void* ids_dev = nullptr;
    int rc = tb_b200_stage_h2d(ids_host, (size_t)n_tokens * sizeof(int32_t), &ids_dev, stream);
    if (rc) return rc;
    rc = tb_b200_embedding(dtype, n_tokens, dim, vocab, static_cast<const int32_t*>(ids_dev), table,
                           y, stream);
    const int rc2 = tb_b200_stage_release(ids_dev, stream);
    return rc ? rc : rc2;
}

// ---------------------------------------------------------------------------
// Allocation-free gather with host ids.
//
// tb_b200_embedding_host_ids stages the caller's host ids in a buffer it
// allocates on the stream and raises range flags in a status word the
// library allocates on first use.  Callers that cannot allocate device
// memory at the point of the call use tb_b200_embedding_host_ids_static
// instead: its scratch is this file-scope device array, which every GPU that
// loads the library holds until the process exits.  Word 0 is the gather
// kernel's status word; the ids follow at a 256-byte offset.
namespace {

constexpr int kStaticIdsOffset = 64;  // int32 words: 256 bytes
static __device__ __align__(256) int32_t
    g_static_scratch[kStaticIdsOffset + TB_B200_STATIC_MAX_TOKENS];

constexpr int kStaticMaxDevices = 64;
int32_t* g_static_dev[kStaticMaxDevices];  // device address of the array, per device
std::mutex g_static_mu;

// Device address of g_static_scratch on the current device (the host-side
// name is only a stand-in).  Looked up once per device.
int static_scratch(int32_t** out) {
    int dev = -1;
    TB_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kStaticMaxDevices) {
        tbh::set_error_text("device ordinal out of range");
        return TB_ERR_DEVICE;
    }
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (g_static_dev[dev] == nullptr) {
        void* p = nullptr;
        TB_CUDA_TRY(cudaGetSymbolAddress(&p, g_static_scratch));
        g_static_dev[dev] = static_cast<int32_t*>(p);
    }
    *out = g_static_dev[dev];
    return TB_OK;
}

}  // namespace

extern "C" int tb_b200_embedding_host_ids_static(int dtype, int64_t n_tokens, int64_t dim,
                                                 int64_t vocab, const int32_t* ids_host,
                                                 const void* table, void* y, void* stream) {
    if (n_tokens < 0 || dim < 0 || vocab < 0) return TB_ERR_INVALID_SHAPE;
    if (n_tokens > TB_B200_STATIC_MAX_TOKENS) {
        tbh::set_error_text(
            "tb_b200_embedding_host_ids_static: n_tokens exceeds TB_B200_STATIC_MAX_TOKENS (65536)");
        return TB_ERR_INVALID_SHAPE;
    }
    if (dtype != TB_DTYPE_F32 && dtype != TB_DTYPE_BF16) return TB_ERR_UNSUPPORTED_DTYPE;
    if (n_tokens == 0 || dim == 0) return TB_OK;
    if (!ids_host || !table || !y) return TB_ERR_INVALID_ARG;
    for (int64_t t = 0; t < n_tokens; ++t)
        if (ids_host[t] < 0 || (int64_t)ids_host[t] >= vocab) return TB_ERR_INVALID_ARG;
    int32_t* scratch = nullptr;
    int rc = static_scratch(&scratch);
    if (rc) return rc;
    cudaStream_t s = tbh::stream_of(stream);
    unsigned int* status = reinterpret_cast<unsigned int*>(scratch);
    int32_t* ids_dev = scratch + kStaticIdsOffset;
    // The array keeps the previous call's contents: the status word restarts at 0.
    TB_CUDA_TRY(cudaMemsetAsync(status, 0, sizeof(unsigned int), s));
    TB_CUDA_TRY(cudaMemcpyAsync(ids_dev, ids_host, (size_t)n_tokens * sizeof(int32_t),
                                cudaMemcpyHostToDevice, s));
    const int64_t row_bytes = dim * (dtype == TB_DTYPE_F32 ? 4 : 2);
    const uintptr_t a = reinterpret_cast<uintptr_t>(table) | reinterpret_cast<uintptr_t>(y);
    if (row_bytes % 16 == 0 && (a & 15) == 0)
        return launch<uint4>(n_tokens, row_bytes, vocab, ids_dev, table, y, status, s);
    if (row_bytes % 4 == 0 && (a & 3) == 0)
        return launch<uint32_t>(n_tokens, row_bytes, vocab, ids_dev, table, y, status, s);
    return launch<uint16_t>(n_tokens, row_bytes, vocab, ids_dev, table, y, status, s);
}
