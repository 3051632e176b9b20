// k_embed_p2p.cu -- the vocab-sharded embedding gather as ONE kernel over
// NVLink: every rank reads its tokens' rows straight out of the owning
// rank's table shard, through CUDA IPC mappings of the other ranks' shards.
//
// The reference engine's embedding is one memcpy per token from a full table
// (src/ops/embedding.c:4-14).  With the table split by vocabulary rows
// across the GPUs of one box (rank r holds rows tb_b200_partition(vocab,
// nranks, r)), the row of token t lives on rank owner(id_t).  The NCCL path
// (comm.cu) packs, exchanges and scatters; here each output row is one plain
// load from the owner's memory -- a peer load over NVLink/NVSwitch when the
// owner is another GPU -- and one store into this rank's output, so the
// gather is a single kernel with no collective, no staging buffer and no
// wait on another GPU: the shards are weights, written once before any
// gather, so nothing on this path depends on another rank's progress.
// Every step is a byte copy: bit-exact with the full-table gather.
//
// Set-up, once per shard: the owner exports an IPC handle of its shard's
// allocation (tb_b200_p2p_export), the handles are exchanged out of band,
// and every other rank opens them (tb_b200_p2p_import) into device
// pointers it passes to the gather.  No multicast and no TMA: plain
// 16-byte loads.
#include <cuda.h>
#include <cuda_runtime.h>
#include <string.h>

#include "tb_internal.h"

namespace {

constexpr int kMaxRanks = 8;
constexpr int kThreads = 256;
constexpr int kBatch = 4;

struct Shards {
    const void* p[kMaxRanks];
};

// Rank owning vocabulary row `id` under tb_b200_partition (the first
// vocab % nranks ranks hold one row more), and that rank's first row.
__device__ __forceinline__ int owner_of(int64_t id, int64_t vocab, int nranks, int64_t& lo) {
    const int64_t base = vocab / nranks, extra = vocab % nranks;
    const int64_t big = extra * (base + 1);
    const int r = id < big ? (int)(id / (base + 1)) : (int)(extra + (id - big) / base);
    lo = (int64_t)r * base + (r < extra ? r : extra);
    return r;
}

// One row per warp, `words` W-words a row.
template <typename W>
__global__ void __launch_bounds__(kThreads)
k_embed_p2p(const int32_t* __restrict__ ids, int64_t n, int64_t vocab, int nranks,
            const __grid_constant__ Shards sh, int64_t words, W* __restrict__ y, unsigned* status) {
    const int64_t j = (int64_t)blockIdx.x * (kThreads / 32) + threadIdx.x / 32;
    if (j >= n) return;
    const int lane = threadIdx.x & 31;
    W* d = y + j * words;
    const int64_t id = ids[j];
    if (id < 0 || id >= vocab) {  // zero the row, raise the flag (never read out of bounds)
        for (int64_t i = lane; i < words; i += 32) d[i] = W{};
        if (lane == 0) atomicOr(status, TB_B200_FLAG_TOKEN_RANGE);
        return;
    }
    int64_t lo;
    const int r = owner_of(id, vocab, nranks, lo);
    const W* s = static_cast<const W*>(sh.p[r]) + (id - lo) * words;
    // kBatch loads in flight per lane before their stores.  Measured level
    // with one at a time on 2 GPUs (0.1166 vs 0.1175 ms at 8192 rows of
    // 16 KB): the gather is bound by NVLink read bandwidth, not latency.
    int64_t i = lane;
    for (; i + 32 * (kBatch - 1) < words; i += 32 * kBatch) {
        W v[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) v[u] = s[i + 32 * u];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) d[i + 32 * u] = v[u];
    }
    for (; i < words; i += 32) d[i] = s[i];
}

using GetRange = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

// cuMemGetAddressRange through the runtime's driver entry point (the
// library links no driver library).
GetRange get_range() {
    static GetRange fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<GetRange>(p);
    }
    return fn;
}

}  // namespace

extern "C" int tb_b200_p2p_export(const void* dev_ptr, void* handle_out, int64_t* offset_out) {
    if (!dev_ptr || !handle_out || !offset_out) return TB_ERR_INVALID_ARG;
    const GetRange range = get_range();
    if (!range) {
        tbh::set_error_text("p2p export: no cuMemGetAddressRange");
        return TB_ERR_DEVICE;
    }
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS) {
        tbh::set_error_text("p2p export: not device memory");
        return TB_ERR_INVALID_ARG;
    }
    cudaIpcMemHandle_t h;
    TB_CUDA_TRY(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
    memcpy(handle_out, &h, sizeof h);
    *offset_out = (int64_t)(reinterpret_cast<uintptr_t>(dev_ptr) - (uintptr_t)base);
    return TB_OK;
}

extern "C" int tb_b200_p2p_import(const void* handle, int64_t offset, void** dev_ptr_out) {
    if (!handle || !dev_ptr_out || offset < 0) return TB_ERR_INVALID_ARG;
    *dev_ptr_out = nullptr;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof h);
    void* base = nullptr;
    TB_CUDA_TRY(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
    *dev_ptr_out = static_cast<char*>(base) + offset;
    return TB_OK;
}

extern "C" int tb_b200_p2p_close(void* dev_ptr, int64_t offset) {
    if (!dev_ptr || offset < 0) return TB_ERR_INVALID_ARG;
    TB_CUDA_TRY(cudaIpcCloseMemHandle(static_cast<char*>(dev_ptr) - offset));
    return TB_OK;
}

extern "C" int tb_b200_embedding_sharded_p2p(int dtype, int64_t n_tokens, int64_t dim,
                                             int64_t vocab, const int32_t* ids,
                                             const void* const* shards, int nranks, void* y,
                                             void* stream) {
    if (n_tokens < 0 || dim < 0 || vocab < 0) return TB_ERR_INVALID_SHAPE;
    if (dtype != TB_DTYPE_F32 && dtype != TB_DTYPE_BF16) return TB_ERR_UNSUPPORTED_DTYPE;
    if (nranks < 1 || nranks > kMaxRanks || vocab < nranks) return TB_ERR_INVALID_ARG;
    if (n_tokens == 0 || dim == 0) return TB_OK;
    if (!ids || !shards || !y) return TB_ERR_INVALID_ARG;
    Shards sh{};
    uintptr_t a = reinterpret_cast<uintptr_t>(y);
    for (int r = 0; r < nranks; ++r) {
        if (!shards[r]) return TB_ERR_INVALID_ARG;
        sh.p[r] = shards[r];
        a |= reinterpret_cast<uintptr_t>(shards[r]);
    }
    tbh::DeviceState* ds = tbh::current_device_state();
    if (!ds) return TB_ERR_DEVICE;
    cudaStream_t s = tbh::stream_of(stream);
    const int64_t row_bytes = dim * (dtype == TB_DTYPE_F32 ? 4 : 2);
    const unsigned grid = (unsigned)((n_tokens + kThreads / 32 - 1) / (kThreads / 32));
    if (row_bytes % 16 == 0 && (a & 15) == 0)
        k_embed_p2p<uint4><<<grid, kThreads, 0, s>>>(ids, n_tokens, vocab, nranks, sh,
                                                     row_bytes / 16, static_cast<uint4*>(y),
                                                     ds->status);
    else if (row_bytes % 4 == 0 && (a & 3) == 0)
        k_embed_p2p<uint32_t><<<grid, kThreads, 0, s>>>(ids, n_tokens, vocab, nranks, sh,
                                                        row_bytes / 4, static_cast<uint32_t*>(y),
                                                        ds->status);
    else
        k_embed_p2p<uint16_t><<<grid, kThreads, 0, s>>>(ids, n_tokens, vocab, nranks, sh,
                                                        row_bytes / 2, static_cast<uint16_t*>(y),
                                                        ds->status);
    TB_LAUNCH_CHECK("p2p embedding kernel");
    return TB_OK;
}
