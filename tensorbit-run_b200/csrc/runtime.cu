// runtime.cu -- device, memory, stream and status entry points of
// libtb_b200.so, plus the host plumbing the kernel files share.
//
// The reference engine has no device layer: its CUDA adapters handed host
// TbTensor data straight to kernels (src/backend/cuda/registry.c:68-78).
// Here device memory is explicit and every kernel entry point is
// asynchronous on a caller-chosen stream.
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>
#include <stdio.h>
#include <string.h>

#include "tb_internal.h"

namespace tbh {

namespace {
thread_local char t_last_error[512] = "";
thread_local cudaStream_t t_stream = nullptr;

constexpr int kMaxDevices = 64;
std::mutex g_mu;
DeviceState g_dev[kMaxDevices];
}  // namespace

void set_error(const char* what, cudaError_t err) {
    snprintf(t_last_error, sizeof t_last_error, "%s: %s (%s)", what, cudaGetErrorName(err),
             cudaGetErrorString(err));
}

void set_error_text(const char* text) { snprintf(t_last_error, sizeof t_last_error, "%s", text); }

cudaStream_t stream_of(void* s) { return s ? static_cast<cudaStream_t>(s) : t_stream; }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

DeviceState* current_device_state() {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        set_error("cudaGetDevice", e);
        return nullptr;
    }
    if (dev < 0 || dev >= kMaxDevices) {
        set_error_text("device ordinal out of range");
        return nullptr;
    }
    DeviceState* ds = &g_dev[dev];
    if (ds->device == dev) return ds;
    std::lock_guard<std::mutex> lock(g_mu);
    if (ds->device == dev) return ds;
    int sms = 0, optin = 0;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) !=
            cudaSuccess) {
        set_error("cudaDeviceGetAttribute", e);
        return nullptr;
    }
    unsigned int* status = nullptr;
    if ((e = cudaMalloc(&status, sizeof(unsigned int))) != cudaSuccess) {
        set_error("cudaMalloc(status)", e);
        return nullptr;
    }
    if ((e = cudaMemset(status, 0, sizeof(unsigned int))) != cudaSuccess) {
        set_error("cudaMemset(status)", e);
        cudaFree(status);
        return nullptr;
    }
    ds->status = status;
    ds->sm_count = sms;
    ds->smem_optin = (size_t)optin;
    ds->device = dev;  // published last: readers test it without the lock
    return ds;
}

namespace {
std::atomic<unsigned long long> g_launches{0};
}

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int ew_grid(int64_t work_items, int threads, const DeviceState* ds, int ctas_per_sm) {
    const int64_t need = (work_items + threads - 1) / threads;
    const int64_t cap = (int64_t)ds->sm_count * ctas_per_sm;
    int64_t g = need < cap ? need : cap;
    return (int)(g < 1 ? 1 : g);
}

}  // namespace tbh

// ====================================================================== C ABI
extern "C" {

int tb_b200_version(void) { return TB_B200_ABI_VERSION; }

const char* tb_b200_last_error(void) { return tbh::t_last_error; }

unsigned long long tb_b200_launch_count(void) {
    return tbh::g_launches.load(std::memory_order_relaxed);
}

int tb_b200_device_count(int* count) {
    if (!count) return TB_ERR_INVALID_ARG;
    *count = 0;
    cudaError_t e = cudaGetDeviceCount(count);
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) {
        cudaGetLastError();
        *count = 0;
        return TB_OK;
    }
    TB_CUDA_TRY(e);
    return TB_OK;
}

int tb_b200_set_device(int device) {
    TB_CUDA_TRY(cudaSetDevice(device));
    return TB_OK;
}

int tb_b200_get_device(int* device) {
    if (!device) return TB_ERR_INVALID_ARG;
    TB_CUDA_TRY(cudaGetDevice(device));
    return TB_OK;
}

int tb_b200_malloc(void** ptr, size_t bytes) {
    if (!ptr) return TB_ERR_INVALID_ARG;
    *ptr = nullptr;
    if (bytes == 0) return TB_OK;
    cudaError_t e = cudaMalloc(ptr, bytes);
    if (e == cudaErrorMemoryAllocation) {
        cudaGetLastError();
        tbh::set_error("cudaMalloc", e);
        return TB_ERR_OOM;
    }
    TB_CUDA_TRY(e);
    return TB_OK;
}

int tb_b200_free(void* ptr) {
    if (ptr) TB_CUDA_TRY(cudaFree(ptr));
    return TB_OK;
}

int tb_b200_malloc_host(void** ptr, size_t bytes) {
    if (!ptr) return TB_ERR_INVALID_ARG;
    *ptr = nullptr;
    if (bytes == 0) return TB_OK;
    TB_CUDA_TRY(cudaMallocHost(ptr, bytes));
    return TB_OK;
}

int tb_b200_free_host(void* ptr) {
    if (ptr) TB_CUDA_TRY(cudaFreeHost(ptr));
    return TB_OK;
}

int tb_b200_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream) {
    if (bytes == 0) return TB_OK;
    if (!dst || !src) return TB_ERR_INVALID_ARG;
    TB_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, tbh::stream_of(stream)));
    return TB_OK;
}

int tb_b200_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream) {
    if (bytes == 0) return TB_OK;
    if (!dst || !src) return TB_ERR_INVALID_ARG;
    TB_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, tbh::stream_of(stream)));
    return TB_OK;
}

int tb_b200_memcpy_d2d(void* dst, const void* src, size_t bytes, void* stream) {
    if (bytes == 0) return TB_OK;
    if (!dst || !src) return TB_ERR_INVALID_ARG;
    TB_CUDA_TRY(
        cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, tbh::stream_of(stream)));
    return TB_OK;
}

int tb_b200_memset(void* dst, int value, size_t bytes, void* stream) {
    if (bytes == 0) return TB_OK;
    if (!dst) return TB_ERR_INVALID_ARG;
    TB_CUDA_TRY(cudaMemsetAsync(dst, value, bytes, tbh::stream_of(stream)));
    return TB_OK;
}

int tb_b200_set_stream(void* stream) {
    tbh::t_stream = static_cast<cudaStream_t>(stream);
    return TB_OK;
}

void* tb_b200_get_stream(void) { return tbh::t_stream; }

int tb_b200_stream_sync(void* stream) {
    TB_CUDA_TRY(cudaStreamSynchronize(tbh::stream_of(stream)));
    return TB_OK;
}

int tb_b200_sync(void) {
    TB_CUDA_TRY(cudaDeviceSynchronize());
    return TB_OK;
}

int tb_b200_is_device_ptr(const void* p, int* is_device) {
    if (!is_device) return TB_ERR_INVALID_ARG;
    *is_device = 0;
    if (!p) return TB_OK;
    cudaPointerAttributes a;
    cudaError_t e = cudaPointerGetAttributes(&a, p);
    if (e != cudaSuccess) {
        // Unregistered host memory on older drivers reports an error.
        cudaGetLastError();
        return TB_OK;
    }
    *is_device = (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) ? 1 : 0;
    return TB_OK;
}

int tb_b200_check_status(void* stream, unsigned int* flags_out) {
    tbh::DeviceState* ds = tbh::current_device_state();
    if (!ds) return TB_ERR_DEVICE;
    cudaStream_t s = tbh::stream_of(stream);
    unsigned int flags = 0;
    TB_CUDA_TRY(cudaMemcpyAsync(&flags, ds->status, sizeof flags, cudaMemcpyDeviceToHost, s));
    TB_CUDA_TRY(cudaMemsetAsync(ds->status, 0, sizeof(unsigned int), s));
    TB_CUDA_TRY(cudaStreamSynchronize(s));
    if (flags_out) *flags_out = flags;
    return flags ? TB_ERR_INVALID_ARG : TB_OK;
}

int tb_b200_partition(int64_t total, int parts, int part, int64_t* lo, int64_t* hi) {
    if (!lo || !hi || total < 0 || parts < 1 || part < 0 || part >= parts)
        return TB_ERR_INVALID_ARG;
    const int64_t base = total / parts, extra = total % parts;
    *lo = part * base + (part < extra ? part : extra);
    *hi = *lo + base + (part < extra ? 1 : 0);
    return TB_OK;
}

}  // extern "C"

extern "C" int tb_b200_stage_h2d(const void* src, size_t bytes, void** dst, void* stream) {
    if (!dst || (!src && bytes)) return TB_ERR_INVALID_ARG;
    *dst = nullptr;
    if (bytes == 0) return TB_OK;
    cudaStream_t s = tbh::stream_of(stream);
    TB_CUDA_TRY(cudaMallocAsync(dst, bytes, s));
    cudaError_t e = cudaMemcpyAsync(*dst, src, bytes, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) {
        tbh::set_error("stage copy", e);
        cudaFreeAsync(*dst, s);
        *dst = nullptr;
        return TB_ERR_DEVICE;
    }
    return TB_OK;
}

extern "C" int tb_b200_stage_release(void* dev, void* stream) {
    if (dev) TB_CUDA_TRY(cudaFreeAsync(dev, tbh::stream_of(stream)));
    return TB_OK;
}
