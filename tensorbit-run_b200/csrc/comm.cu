// comm.cu -- NCCL communicator and the vocab-sharded embedding gather.
//
// The reference engine is single-process and has no communication layer;
// its embedding is one memcpy per token from a full table
// (src/ops/embedding.c:4-14).  At a 128K vocabulary the table is split by
// vocabulary rows across the GPUs of one box while the token rows are split
// by position, so a token's row usually lives on another GPU.  Each rank:
//   1. builds, on the host, the exchange plan from the replicated ids:
//      which of its table rows every other rank needs (in token order) and
//      where the rows it receives go in its output (tb_b200_shard_plan);
//   2. gathers the rows it owns: its own tokens' rows straight into its
//      output, other ranks' rows into one packed send buffer (one kernel);
//   3. exchanges packed rows with every peer in one grouped NCCL
//      send/recv (NVLink/NVSwitch), only rows that are needed;
//   4. scatters the received rows into its output (one kernel).
// Every step is a byte copy, so the result is bit-exact with the
// full-table gather.  The communicator is created non-blocking, and every
// host-side wait on it is bounded (TB_B200_COMM_TIMEOUT_S seconds, default
// 120): creation, and the enqueue of the grouped exchange.  The exchange
// itself runs later on the stream, where an NCCL kernel waits for its peers;
// tb_b200_comm_wait bounds that wait too: it polls the stream's progress and
// the communicator's error state, and on timeout aborts the communicator
// (which ends its kernels) and returns TB_ERR_DEVICE.  A rank that never
// arrives thus makes the others fail instead of hanging.
//
// NCCL is not linked: its entry points are resolved with dlopen/dlsym on
// first use.  A process that also loads PyTorch then shares torch's NCCL
// (dlopen of the soname returns the library already loaded), instead of a
// second libnccl.so.2 claiming the soname before torch's and breaking it.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <nccl_device.h>

#include <mutex>

#include <chrono>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <thread>
#include <vector>

#include "tb_internal.h"

namespace {

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*);
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*);
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*);
    ncclResult_t (*CommAbort)(ncclComm_t);
    ncclResult_t (*CommFinalize)(ncclComm_t);
    ncclResult_t (*CommDestroy)(ncclComm_t);
    const char* (*GetErrorString)(ncclResult_t);
    ncclResult_t (*GroupStart)();
    ncclResult_t (*GroupEnd)();
    ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    // symmetric memory windows (NCCL 2.27+); null when the NCCL has none
    ncclResult_t (*MemAlloc)(void**, size_t);
    ncclResult_t (*MemFree)(void*);
    ncclResult_t (*WindowRegister)(ncclComm_t, void*, size_t, ncclWindow_t*, int);
    ncclResult_t (*WindowDeregister)(ncclComm_t, ncclWindow_t);
};

NcclApi g_nccl;
bool g_nccl_ok = false;
std::once_flag g_nccl_once;

// Resolve NCCL once; false (with the error text set) if it is unavailable.
bool nccl_api() {
    std::call_once(g_nccl_once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        bool ok = true;
        auto sym = [&](auto& fp, const char* name) {
            *reinterpret_cast<void**>(&fp) = dlsym(h, name);
            ok = ok && fp != nullptr;
        };
        sym(g_nccl.GetUniqueId, "ncclGetUniqueId");
        sym(g_nccl.CommInitRankConfig, "ncclCommInitRankConfig");
        sym(g_nccl.CommGetAsyncError, "ncclCommGetAsyncError");
        sym(g_nccl.CommAbort, "ncclCommAbort");
        sym(g_nccl.CommFinalize, "ncclCommFinalize");
        sym(g_nccl.CommDestroy, "ncclCommDestroy");
        sym(g_nccl.GetErrorString, "ncclGetErrorString");
        sym(g_nccl.GroupStart, "ncclGroupStart");
        sym(g_nccl.GroupEnd, "ncclGroupEnd");
        sym(g_nccl.Send, "ncclSend");
        sym(g_nccl.Recv, "ncclRecv");
        g_nccl_ok = ok;
        *reinterpret_cast<void**>(&g_nccl.MemAlloc) = dlsym(h, "ncclMemAlloc");
        *reinterpret_cast<void**>(&g_nccl.MemFree) = dlsym(h, "ncclMemFree");
        *reinterpret_cast<void**>(&g_nccl.WindowRegister) = dlsym(h, "ncclCommWindowRegister");
        *reinterpret_cast<void**>(&g_nccl.WindowDeregister) = dlsym(h, "ncclCommWindowDeregister");
    });
    if (!g_nccl_ok) tbh::set_error_text("NCCL (libnccl.so.2) could not be loaded");
    return g_nccl_ok;
}

ncclComm_t g_comm = nullptr;
int g_rank = 0, g_nranks = 0;

double timeout_s() {
    const char* e = getenv("TB_B200_COMM_TIMEOUT_S");
    const double v = e ? atof(e) : 0.0;
    return v > 0 ? v : 120.0;
}

void nccl_error(const char* what, ncclResult_t r) {
    char buf[384];
    snprintf(buf, sizeof buf, "%s: %s", what, g_nccl.GetErrorString(r));
    tbh::set_error_text(buf);
}

// Wait until the non-blocking communicator finished the last call.
int wait_comm(const char* what) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        ncclResult_t r = g_nccl.CommGetAsyncError(g_comm, &st);
        if (r != ncclSuccess) {
            nccl_error(what, r);
            return TB_ERR_DEVICE;
        }
        if (st == ncclSuccess) return TB_OK;
        if (st != ncclInProgress) {
            nccl_error(what, st);
            g_nccl.CommAbort(g_comm);
            g_comm = nullptr;
            return TB_ERR_DEVICE;
        }
        const double el =
            std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (el > timeout_s()) {
            tbh::set_error_text("NCCL call timed out; communicator aborted");
            g_nccl.CommAbort(g_comm);
            g_comm = nullptr;
            return TB_ERR_DEVICE;
        }
        if (el > 1e-3)
            std::this_thread::sleep_for(std::chrono::microseconds(50));
        else
            std::this_thread::yield();
    }
}

// Copy n rows of `words` W-words: dst[drow(j)] = src[srow(j)], where a NULL
// index list means the identity.  64 threads per row, four loads in flight
// per thread before their stores.
template <typename W>
__global__ void __launch_bounds__(256)
k_rows(W* __restrict__ dst, const int32_t* __restrict__ drow, const W* __restrict__ src,
       const int32_t* __restrict__ srow, int64_t n, int64_t words) {
    constexpr int kGroup = 64, kU = 4;
    const int64_t j = (int64_t)blockIdx.x * (blockDim.x / kGroup) + threadIdx.x / kGroup;
    if (j >= n) return;
    const int64_t di = drow ? drow[j] : j, si = srow ? srow[j] : j;
    const W* s = src + si * words;
    W* d = dst + di * words;
    int64_t i = threadIdx.x % kGroup;
    for (; i + (kU - 1) * kGroup < words; i += kU * kGroup) {
        W v[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) v[u] = s[i + u * kGroup];
#pragma unroll
        for (int u = 0; u < kU; ++u) d[i + u * kGroup] = v[u];
    }
    for (; i < words; i += kGroup) d[i] = s[i];
}

int copy_rows(void* dst, const int32_t* drow, const void* src, const int32_t* srow, int64_t n,
              int64_t row_bytes, cudaStream_t s) {
    if (n == 0) return TB_OK;
    const unsigned grid = (unsigned)((n + 3) / 4);
    const uintptr_t a = reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src);
    if (row_bytes % 16 == 0 && (a & 15) == 0)
        k_rows<uint4><<<grid, 256, 0, s>>>(static_cast<uint4*>(dst), drow,
                                           static_cast<const uint4*>(src), srow, n, row_bytes / 16);
    else if (row_bytes % 4 == 0 && (a & 3) == 0)
        k_rows<uint32_t><<<grid, 256, 0, s>>>(static_cast<uint32_t*>(dst), drow,
                                              static_cast<const uint32_t*>(src), srow, n,
                                              row_bytes / 4);
    else
        k_rows<uint16_t><<<grid, 256, 0, s>>>(static_cast<uint16_t*>(dst), drow,
                                              static_cast<const uint16_t*>(src), srow, n,
                                              row_bytes / 2);
    TB_LAUNCH_CHECK("row copy kernel");
    return TB_OK;
}

// Rank owning table row `id` under tb_b200_partition(vocab, nranks, .):
// ends[r] is rank r's end row; a short linear search (nranks <= 8 on a box).
inline int owner_of(int64_t id, const int64_t* ends, int nranks) {
    int r = 0;
    while (r < nranks - 1 && id >= ends[r]) ++r;
    return r;
}

// Per-communicator buffers of the sharded gather, kept across calls: the
// device block [plan indices | send rows | receive rows], grown on demand,
// and a ring of two page-locked plan buffers for the host-to-device copy.
struct GatherBufs {
    void* dev = nullptr;
    size_t dev_cap = 0;
    int32_t* host[2] = {nullptr, nullptr};
    size_t host_cap[2] = {0, 0};
    cudaEvent_t host_free[2] = {nullptr, nullptr};  // the copy out of host[k] is done
    cudaEvent_t dev_free = nullptr;                 // the last call is done with `dev`
    int k = 0;
};
GatherBufs g_bufs;

// Wait for `ev` at most TB_B200_COMM_TIMEOUT_S; false on timeout or error.
bool wait_event(cudaEvent_t ev) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t e = cudaEventQuery(ev);
        if (e == cudaSuccess) return true;
        if (e != cudaErrorNotReady) return false;
        if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() >
            timeout_s())
            return false;
        std::this_thread::yield();
    }
}

void release_bufs() {
    // The buffers may still be used by queued work: wait for it, bounded.
    // Work that never finishes (an exchange with a peer that is gone, not
    // ended by an abort) keeps its buffers: they are left allocated.
    bool idle = true;
    if (g_bufs.dev_free) idle = wait_event(g_bufs.dev_free);
    for (int k = 0; k < 2; ++k)
        if (g_bufs.host_free[k]) idle = wait_event(g_bufs.host_free[k]) && idle;
    if (!idle) {
        g_bufs = GatherBufs();
        return;
    }
    for (int k = 0; k < 2; ++k) {
        if (g_bufs.host[k]) cudaFreeHost(g_bufs.host[k]);
        if (g_bufs.host_free[k]) cudaEventDestroy(g_bufs.host_free[k]);
        g_bufs.host[k] = nullptr;
        g_bufs.host_cap[k] = 0;
        g_bufs.host_free[k] = nullptr;
    }
    if (g_bufs.dev) cudaFree(g_bufs.dev);
    if (g_bufs.dev_free) cudaEventDestroy(g_bufs.dev_free);
    g_bufs = GatherBufs();
}

// Symmetric windows made by tb_b200_comm_window_alloc on this process's
// communicator: NCCL maps every rank's window of a registration into this
// GPU's address space, so a peer's bytes are a plain load away.
struct WinRec {
    char* ptr;
    size_t bytes;
    ncclWindow_t win;
};
std::vector<WinRec> g_wins;

// One row per warp: row j of y is row ids[j] of the full table, read from
// its owner's shard through the window (a peer load over NVLink/NVSwitch
// when the owner is another GPU).  Every rank's shard sits at byte `base`
// of its window.  Ids outside [0, vocab) zero the row and raise the flag.
template <typename W>
__global__ void __launch_bounds__(256)
k_embed_window(const int32_t* __restrict__ ids, int64_t n, int64_t vocab, int nranks,
               ncclWindow_t win, size_t base, int64_t words, W* __restrict__ y,
               unsigned* status) {
    constexpr int kBatch = 4;
    const int64_t j = (int64_t)blockIdx.x * 8 + threadIdx.x / 32;
    if (j >= n) return;
    const int lane = threadIdx.x & 31;
    W* d = y + j * words;
    const int64_t id = ids[j];
    if (id < 0 || id >= vocab) {
        for (int64_t i = lane; i < words; i += 32) d[i] = W{};
        if (lane == 0) atomicOr(status, TB_B200_FLAG_TOKEN_RANGE);
        return;
    }
    const int64_t pb = vocab / nranks, extra = vocab % nranks, big = extra * (pb + 1);
    const int r = id < big ? (int)(id / (pb + 1)) : (int)(extra + (id - big) / pb);
    const int64_t lo = (int64_t)r * pb + (r < extra ? r : extra);
    const W* s = static_cast<const W*>(
        ncclGetPeerPointer(win, base + (size_t)((id - lo) * words) * sizeof(W), r));
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

bool have_windows() {
    return g_nccl.MemAlloc && g_nccl.MemFree && g_nccl.WindowRegister && g_nccl.WindowDeregister;
}

}  // namespace

extern "C" {

int tb_b200_shard_plan(int64_t n_tokens, int64_t vocab, int nranks, int rank,
                       const int32_t* ids, int64_t* send_counts, int64_t* recv_counts,
                       int32_t* send_rows, int32_t* recv_rows, int32_t* local_dst,
                       int32_t* local_src, int64_t* n_local) {
    if (n_tokens < 0 || vocab < nranks || nranks < 1 || rank < 0 || rank >= nranks)
        return TB_ERR_INVALID_ARG;
    if (!send_counts || !recv_counts || !send_rows || !recv_rows || !local_dst || !local_src ||
        !n_local || (n_tokens && !ids))
        return TB_ERR_INVALID_ARG;
    for (int64_t t = 0; t < n_tokens; ++t)
        if (ids[t] < 0 || ids[t] >= vocab) return TB_ERR_INVALID_ARG;
    // One pass over the tokens: each token's owner from the vocab parts'
    // boundaries (no division per token).
    int64_t vend[64], tend[64];
    if (nranks > 64) return TB_ERR_INVALID_ARG;
    for (int r = 0; r < nranks; ++r) {
        int64_t lo;
        tb_b200_partition(vocab, nranks, r, &lo, &vend[r]);
        tb_b200_partition(n_tokens, nranks, r, &lo, &tend[r]);
    }
    const int64_t my_vlo = rank ? vend[rank - 1] : 0;
    const int64_t my_tlo = rank ? tend[rank - 1] : 0, my_thi = tend[rank];
    int64_t ns = 0, nl = 0;
    // Rows this rank sends: destination-major (destinations own consecutive
    // token parts), token order within a destination.
    int d = 0;
    for (int r = 0; r < nranks; ++r) send_counts[r] = recv_counts[r] = 0;
    for (int64_t t = 0; t < n_tokens; ++t) {
        while (t >= tend[d]) ++d;
        const int64_t id = ids[t];
        if (owner_of(id, vend, nranks) != rank) continue;
        if (d == rank) {
            local_dst[nl] = (int32_t)(t - my_tlo);
            local_src[nl] = (int32_t)(id - my_vlo);
            ++nl;
        } else {
            send_rows[ns++] = (int32_t)(id - my_vlo);
            ++send_counts[d];
        }
    }
    // Rows this rank receives: source-major, token order within a source
    // (a counting sort of this rank's tokens by owner).
    int64_t start[65];
    for (int64_t t = my_tlo; t < my_thi; ++t) {
        const int o = owner_of(ids[t], vend, nranks);
        if (o != rank) ++recv_counts[o];
    }
    start[0] = 0;
    for (int r = 0; r < nranks; ++r) start[r + 1] = start[r] + recv_counts[r];
    for (int64_t t = my_tlo; t < my_thi; ++t) {
        const int o = owner_of(ids[t], vend, nranks);
        if (o != rank) recv_rows[start[o]++] = (int32_t)(t - my_tlo);
    }
    *n_local = nl;
    return TB_OK;
}

int tb_b200_comm_unique_id(void* id_out) {
    if (!id_out) return TB_ERR_INVALID_ARG;
    if (!nccl_api()) return TB_ERR_DEVICE;
    static_assert(sizeof(ncclUniqueId) == TB_B200_COMM_ID_BYTES, "NCCL id size");
    ncclUniqueId id;
    ncclResult_t r = g_nccl.GetUniqueId(&id);
    if (r != ncclSuccess) {
        nccl_error("ncclGetUniqueId", r);
        return TB_ERR_DEVICE;
    }
    memcpy(id_out, &id, sizeof id);
    return TB_OK;
}

int tb_b200_comm_init(int nranks, int rank, const void* unique_id, int device) {
    if (nranks < 1 || rank < 0 || rank >= nranks || !unique_id) return TB_ERR_INVALID_ARG;
    if (g_comm) return TB_ERR_INVALID_ARG;  // one communicator per process
    if (!nccl_api()) return TB_ERR_DEVICE;
    TB_CUDA_TRY(cudaSetDevice(device));
    ncclUniqueId id;
    memcpy(&id, unique_id, sizeof id);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = g_nccl.CommInitRankConfig(&g_comm, nranks, id, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        nccl_error("ncclCommInitRankConfig", r);
        g_comm = nullptr;
        return TB_ERR_DEVICE;
    }
    const int rc = wait_comm("ncclCommInitRankConfig");
    if (rc) return rc;
    g_rank = rank;
    g_nranks = nranks;
    release_bufs();  // left from an aborted communicator, if any
    TB_CUDA_TRY(cudaEventCreateWithFlags(&g_bufs.dev_free, cudaEventDisableTiming));
    for (int k = 0; k < 2; ++k)
        TB_CUDA_TRY(cudaEventCreateWithFlags(&g_bufs.host_free[k], cudaEventDisableTiming));
    return TB_OK;
}

int tb_b200_comm_destroy(void) {
    release_bufs();
    if (!g_comm) {
        g_wins.clear();  // an aborted communicator took its windows with it
        return TB_OK;
    }
    while (!g_wins.empty())  // every rank destroys: deregister in allocation order
        tb_b200_comm_window_free(g_wins.front().ptr);  // (drops the record first)
    ncclResult_t r = g_nccl.CommFinalize(g_comm);
    int rc = TB_OK;
    if (r != ncclSuccess && r != ncclInProgress) {
        nccl_error("ncclCommFinalize", r);
        rc = TB_ERR_DEVICE;
    } else {
        rc = wait_comm("ncclCommFinalize");
    }
    if (g_comm) g_nccl.CommDestroy(g_comm);
    g_comm = nullptr;
    g_rank = 0;
    g_nranks = 0;
    return rc;
}

int tb_b200_comm_wait(void* stream) {
    if (!g_comm) {
        tbh::set_error_text("tb_b200_comm_wait: no communicator (tb_b200_comm_init)");
        return TB_ERR_INVALID_ARG;
    }
    cudaStream_t s = tbh::stream_of(stream);
    cudaEvent_t ev = nullptr;
    TB_CUDA_TRY(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    cudaError_t e = cudaEventRecord(ev, s);
    if (e != cudaSuccess) {
        cudaEventDestroy(ev);
        tbh::set_error("tb_b200_comm_wait: event record", e);
        return TB_ERR_DEVICE;
    }
    const double limit = timeout_s();
    const auto t0 = std::chrono::steady_clock::now();
    auto elapsed = [&]() {
        return std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    };
    int rc = TB_OK;
    for (;;) {
        e = cudaEventQuery(ev);
        if (e == cudaSuccess) break;
        if (e != cudaErrorNotReady) {
            tbh::set_error("tb_b200_comm_wait", e);
            rc = TB_ERR_DEVICE;
            break;
        }
        ncclResult_t st = ncclSuccess;
        const ncclResult_t r = g_nccl.CommGetAsyncError(g_comm, &st);
        const bool failed = r != ncclSuccess || (st != ncclSuccess && st != ncclInProgress);
        if (failed || elapsed() > limit) {
            if (failed)
                nccl_error("tb_b200_comm_wait", r != ncclSuccess ? r : st);
            else
                tbh::set_error_text("tb_b200_comm_wait: exchange timed out; communicator aborted");
            // Aborting ends the communicator's kernels still waiting for
            // peers, so the stream drains; wait for that, bounded again.
            g_nccl.CommAbort(g_comm);
            g_comm = nullptr;
            g_rank = 0;
            g_nranks = 0;
            const auto t1 = std::chrono::steady_clock::now();
            while (cudaEventQuery(ev) == cudaErrorNotReady &&
                   std::chrono::duration<double>(std::chrono::steady_clock::now() - t1).count() <
                       limit)
                std::this_thread::sleep_for(std::chrono::microseconds(200));
            rc = TB_ERR_DEVICE;
            break;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
    cudaEventDestroy(ev);
    return rc;
}

int tb_b200_comm_info(int* rank, int* nranks) {
    if (!rank || !nranks) return TB_ERR_INVALID_ARG;
    *rank = g_comm ? g_rank : 0;
    *nranks = g_comm ? g_nranks : 0;
    return TB_OK;
}

int tb_b200_embedding_sharded(int dtype, int64_t n_tokens, int64_t dim, int64_t vocab,
                              const int32_t* ids, const void* table_shard, void* y_local,
                              void* stream) {
    if (!g_comm) {
        tbh::set_error_text("tb_b200_embedding_sharded: no communicator (tb_b200_comm_init)");
        return TB_ERR_INVALID_ARG;
    }
    if (dtype != TB_DTYPE_F32 && dtype != TB_DTYPE_BF16) return TB_ERR_UNSUPPORTED_DTYPE;
    if (n_tokens < 0 || dim < 0 || vocab < g_nranks || n_tokens > INT32_MAX)
        return TB_ERR_INVALID_SHAPE;
    if (n_tokens && (!ids || !table_shard)) return TB_ERR_INVALID_ARG;
    const int N = g_nranks, me = g_rank;
    const int64_t row_bytes = dim * (dtype == TB_DTYPE_F32 ? 4 : 2);
    int64_t tlo, thi;
    tb_b200_partition(n_tokens, N, me, &tlo, &thi);
    if (thi > tlo && !y_local) return TB_ERR_INVALID_ARG;

    // Plan on the host, straight into a page-locked buffer of the ring:
    // [send rows | recv rows | local dst | local src], each of capacity
    // n_tokens, copied to the device block in one transfer.
    GatherBufs& B = g_bufs;
    const int k = B.k;
    B.k ^= 1;
    const size_t idx_ints = 4 * (size_t)n_tokens + 4;
    cudaError_t e = wait_event(B.host_free[k]) ? cudaSuccess : cudaErrorNotReady;  // its copy two calls ago
    if (e == cudaSuccess && B.host_cap[k] < idx_ints) {
        if (B.host[k]) cudaFreeHost(B.host[k]);
        B.host[k] = nullptr;
        B.host_cap[k] = 0;
        e = cudaMallocHost(reinterpret_cast<void**>(&B.host[k]), idx_ints * sizeof(int32_t));
        if (e == cudaSuccess) B.host_cap[k] = idx_ints;
    }
    if (e != cudaSuccess) {
        tbh::set_error("sharded embedding plan buffer", e);
        return TB_ERR_DEVICE;
    }
    std::vector<int64_t> sc(N), rcnt(N);
    int32_t* send_rows = B.host[k];
    int32_t* recv_rows = send_rows + n_tokens;
    int32_t* ldst = recv_rows + n_tokens;
    int32_t* lsrc = ldst + n_tokens;
    int64_t nl = 0;
    int rc = tb_b200_shard_plan(n_tokens, vocab, N, me, ids, sc.data(), rcnt.data(), send_rows,
                                recv_rows, ldst, lsrc, &nl);
    if (rc) return rc;
    int64_t ns = 0, nr = 0;
    for (int p = 0; p < N; ++p) {
        ns += sc[p];
        nr += rcnt[p];
    }
    // Device block: the four index lists at their fixed offsets, then the
    // send rows and the received rows (16-byte aligned).
    const size_t idx_bytes = (idx_ints * sizeof(int32_t) + 255) / 256 * 256;
    const size_t send_bytes = ((size_t)(ns * row_bytes) + 255) / 256 * 256;
    const size_t need = idx_bytes + send_bytes + (size_t)(nr * row_bytes);
    cudaStream_t s = tbh::stream_of(stream);
    if (B.dev_cap < need) {  // grow: the previous call must be done with the block
        e = wait_event(B.dev_free) ? cudaSuccess : cudaErrorNotReady;
        if (e == cudaSuccess) {
            if (B.dev) cudaFree(B.dev);
            B.dev = nullptr;
            B.dev_cap = 0;
            e = cudaMalloc(&B.dev, need + need / 4);
            if (e == cudaSuccess) B.dev_cap = need + need / 4;
        }
        if (e != cudaSuccess) {
            tbh::set_error("sharded embedding buffers", e);
            return TB_ERR_DEVICE;
        }
    }
    // A call on another stream may still be using the block.
    TB_CUDA_TRY(cudaStreamWaitEvent(s, B.dev_free, 0));
    int32_t* d_idx = static_cast<int32_t*>(B.dev);
    TB_CUDA_TRY(cudaMemcpyAsync(d_idx, B.host[k], idx_ints * sizeof(int32_t),
                                cudaMemcpyHostToDevice, s));
    TB_CUDA_TRY(cudaEventRecord(B.host_free[k], s));
    const int32_t* d_send = d_idx;
    const int32_t* d_recv = d_idx + n_tokens;
    const int32_t* d_ldst = d_recv + n_tokens;
    const int32_t* d_lsrc = d_ldst + n_tokens;
    char* sendbuf = static_cast<char*>(B.dev) + idx_bytes;
    char* recvbuf = sendbuf + send_bytes;
    // Own rows: local tokens straight to the output, others packed.
    if ((rc = copy_rows(y_local, d_ldst, table_shard, d_lsrc, nl, row_bytes, s)) ||
        (rc = copy_rows(sendbuf, nullptr, table_shard, d_send, ns, row_bytes, s)))
        return rc;
    // One grouped exchange with every peer.
    ncclResult_t r = ncclSuccess;
    if (N > 1) {
        r = g_nccl.GroupStart();
        int64_t so = 0, ro = 0;
        for (int p = 0; p < N && r == ncclSuccess; ++p) {
            if (p == me) continue;
            if (sc[p])
                r = g_nccl.Send(sendbuf + so * row_bytes, (size_t)(sc[p] * row_bytes), ncclUint8, p,
                                g_comm, s);
            if ((r == ncclSuccess || r == ncclInProgress) && rcnt[p])
                r = g_nccl.Recv(recvbuf + ro * row_bytes, (size_t)(rcnt[p] * row_bytes), ncclUint8,
                                p, g_comm, s);
            if (r == ncclInProgress) r = ncclSuccess;
            so += sc[p];
            ro += rcnt[p];
        }
        ncclResult_t r2 = g_nccl.GroupEnd();
        if (r == ncclSuccess && r2 != ncclSuccess && r2 != ncclInProgress) r = r2;
        if (r != ncclSuccess) {
            nccl_error("sharded embedding exchange", r);
            return TB_ERR_DEVICE;
        }
        rc = wait_comm("sharded embedding exchange");
        if (rc) return rc;
    }
    rc = copy_rows(y_local, d_recv, recvbuf, nullptr, nr, row_bytes, s);
    if (rc) return rc;
    TB_CUDA_TRY(cudaEventRecord(B.dev_free, s));
    return TB_OK;
}

int tb_b200_comm_window_alloc(size_t bytes, void** ptr) {
    if (!ptr || !bytes) return TB_ERR_INVALID_ARG;
    *ptr = nullptr;
    if (!g_comm) {
        tbh::set_error_text("tb_b200_comm_window_alloc: no communicator (tb_b200_comm_init)");
        return TB_ERR_INVALID_ARG;
    }
    if (!have_windows()) {
        tbh::set_error_text("the loaded NCCL has no symmetric memory windows");
        return TB_ERR_DEVICE;
    }
    bytes = (bytes + NCCL_WIN_REQUIRED_ALIGNMENT - 1) / NCCL_WIN_REQUIRED_ALIGNMENT *
            NCCL_WIN_REQUIRED_ALIGNMENT;
    void* p = nullptr;
    ncclResult_t r = g_nccl.MemAlloc(&p, bytes);
    if (r != ncclSuccess) {
        nccl_error("ncclMemAlloc", r);
        return TB_ERR_DEVICE;
    }
    ncclWindow_t w = nullptr;
    r = g_nccl.WindowRegister(g_comm, p, bytes, &w, NCCL_WIN_COLL_SYMMETRIC);
    if (r != ncclSuccess && r != ncclInProgress) {
        nccl_error("ncclCommWindowRegister", r);
        g_nccl.MemFree(p);
        return TB_ERR_DEVICE;
    }
    const int rc = wait_comm("ncclCommWindowRegister");
    if (rc) {
        if (g_comm) g_nccl.MemFree(p);  // after an abort the memory went with the communicator
        return rc;
    }
    g_wins.push_back(WinRec{static_cast<char*>(p), bytes, w});
    *ptr = p;
    return TB_OK;
}

int tb_b200_comm_window_free(void* ptr) {
    if (!ptr) return TB_OK;
    for (size_t i = 0; i < g_wins.size(); ++i) {
        if (g_wins[i].ptr != ptr) continue;
        const WinRec w = g_wins[i];
        g_wins.erase(g_wins.begin() + (ptrdiff_t)i);
        if (!g_comm) return TB_OK;
        ncclResult_t r = g_nccl.WindowDeregister(g_comm, w.win);
        int rc = TB_OK;
        if (r != ncclSuccess && r != ncclInProgress) {
            nccl_error("ncclCommWindowDeregister", r);
            rc = TB_ERR_DEVICE;
        } else {
            rc = wait_comm("ncclCommWindowDeregister");
        }
        if (rc == TB_OK) {
            r = g_nccl.MemFree(w.ptr);
            if (r != ncclSuccess) {
                nccl_error("ncclMemFree", r);
                rc = TB_ERR_DEVICE;
            }
        }
        return rc;
    }
    return TB_ERR_INVALID_ARG;
}

int tb_b200_embedding_sharded_window(int dtype, int64_t n_tokens, int64_t dim, int64_t vocab,
                                     const int32_t* ids, const void* shard, void* y,
                                     void* stream) {
    if (!g_comm) {
        tbh::set_error_text("tb_b200_embedding_sharded_window: no communicator");
        return TB_ERR_INVALID_ARG;
    }
    if (dtype != TB_DTYPE_F32 && dtype != TB_DTYPE_BF16) return TB_ERR_UNSUPPORTED_DTYPE;
    if (n_tokens < 0 || dim < 0 || vocab < g_nranks) return TB_ERR_INVALID_SHAPE;
    if (n_tokens == 0 || dim == 0) return TB_OK;
    if (!ids || !shard || !y) return TB_ERR_INVALID_ARG;
    const WinRec* w = nullptr;
    for (const WinRec& r : g_wins)
        if (static_cast<const char*>(shard) >= r.ptr &&
            static_cast<const char*>(shard) < r.ptr + r.bytes)
            w = &r;
    if (!w) {
        tbh::set_error_text("tb_b200_embedding_sharded_window: shard is not in a window");
        return TB_ERR_INVALID_ARG;
    }
    const int64_t row_bytes = dim * (dtype == TB_DTYPE_F32 ? 4 : 2);
    const size_t base = (size_t)(static_cast<const char*>(shard) - w->ptr);
    int64_t lo, hi;
    tb_b200_partition(vocab, g_nranks, g_rank, &lo, &hi);
    if (base + (size_t)((hi - lo) * row_bytes) > w->bytes) return TB_ERR_INVALID_SHAPE;
    const tbh::DeviceState* ds = tbh::current_device_state();
    if (!ds) return TB_ERR_DEVICE;
    cudaStream_t s = tbh::stream_of(stream);
    const unsigned grid = (unsigned)((n_tokens + 7) / 8);
    const uintptr_t a = reinterpret_cast<uintptr_t>(y) | (uintptr_t)base | (uintptr_t)row_bytes;
    if ((a & 15) == 0)
        k_embed_window<uint4><<<grid, 256, 0, s>>>(ids, n_tokens, vocab, g_nranks, w->win, base,
                                                   row_bytes / 16, static_cast<uint4*>(y),
                                                   ds->status);
    else if ((a & 3) == 0)
        k_embed_window<uint32_t><<<grid, 256, 0, s>>>(ids, n_tokens, vocab, g_nranks, w->win,
                                                      base, row_bytes / 4,
                                                      static_cast<uint32_t*>(y), ds->status);
    else
        k_embed_window<uint16_t><<<grid, 256, 0, s>>>(ids, n_tokens, vocab, g_nranks, w->win,
                                                      base, row_bytes / 2,
                                                      static_cast<uint16_t*>(y), ds->status);
    TB_LAUNCH_CHECK("sharded embedding kernel (window)");
    return TB_OK;
}

}  // extern "C"
