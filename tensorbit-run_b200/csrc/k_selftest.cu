// k_selftest.cu -- a check that the library's bounded device waits end.
//
// The staged kernels wait on shared-memory mbarriers for their bulk copies
// (tma.cuh).  Every such wait is bounded by %globaltimer: when the bound
// runs out the waiter raises TB_B200_FLAG_WAIT_TIMEOUT in the device status
// word and the kernel returns, so a lost copy costs a wrong result and a
// flag, never a hung GPU.  This entry point runs that same wait on one
// mbarrier in a one-warp kernel:
//   supply != 0: one 16-byte bulk copy completes the barrier's expected
//                bytes -- the wait ends normally, no flag;
//   supply == 0: the barrier expects 16 bytes that no copy brings -- the
//                wait gives up after limit_us, raises the flag and returns.
// No copy is ever in flight when the kernel exits.  The reference has no
// device code of this kind.
#include <cuda_runtime.h>

#include "tb_internal.h"
#include "tma.cuh"

namespace {

// A 16-byte aligned global source for the supplied copy.
__device__ __align__(16) uint32_t g_selftest_src[4] = {1u, 2u, 3u, 4u};

__global__ void __launch_bounds__(32)
k_wait_selftest(int supply, uint64_t limit_ns, unsigned int* status) {
    __shared__ __align__(16) uint32_t dst[4];
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        tbk::mbar_init(&bar, 1);
        tbk::fence_mbar_init();
    }
    __syncwarp();
    if (threadIdx.x == 0) {
        tbk::mbar_expect_tx(&bar, sizeof dst);  // the one arrival, plus 16 bytes to come
        if (supply) tbk::bulk_g2s(dst, g_selftest_src, sizeof dst, &bar);
    }
    __syncwarp();
    const bool done = tbk::mbar_wait(&bar, 0, status, limit_ns);
    // A completed copy must have brought the source's words.
    if (done && threadIdx.x < 4 && dst[threadIdx.x] != threadIdx.x + 1u)
        atomicOr(status, tbk::kFlagTimeout);
}

}  // namespace

extern "C" int tb_b200_selftest_wait(int supply, uint32_t limit_us, void* stream) {
    if (limit_us == 0 || limit_us > 1000000u) return TB_ERR_INVALID_ARG;
    tbh::DeviceState* ds = tbh::current_device_state();
    if (!ds) return TB_ERR_DEVICE;
    k_wait_selftest<<<1, 32, 0, tbh::stream_of(stream)>>>(supply, (uint64_t)limit_us * 1000ull,
                                                           ds->status);
    TB_LAUNCH_CHECK("wait self-test kernel");
    return TB_OK;
}
