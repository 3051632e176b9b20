// k_elementwise.cu -- SiLU, tanh-GELU, SwiGLU and residual add over n
// elements (reference arithmetic at ew_apply, bodies.cuh).
//
// Data path: HBM bound (2 or 3 * n * s bytes).  A grid-stride loop over
// 16-byte vectors, sized to fill the SMs: one vector per thread per round
// for SiLU/GELU/SwiGLU (their expf/tanhf and division make register count
// and occupancy the limit), four for the residual add.  A ragged tail
// (n not a multiple of the vector width) goes to a one-CTA scalar launch;
// unaligned pointers use the scalar instantiation throughout.
#include "bodies.cuh"
#include "tb_internal.h"

namespace {

using tbk::Elt;

template <typename T, int VEC, int OP, int UNROLL>
__global__ void __launch_bounds__(256, 4)
k_ew(const T* a, const T* b, T* out, int64_t nvec) {
    tbk::ew_body<T, VEC, OP, UNROLL>(a, b, out, nvec, blockIdx.x, gridDim.x);
}

template <typename T, int OP>
int launch(const void* a, const void* b, void* out, int64_t n, cudaStream_t s) {
    tbh::DeviceState* ds = tbh::current_device_state();
    if (!ds) return TB_ERR_DEVICE;
    constexpr int V = Elt<T>::kVec;
    // Transcendental ops issue enough arithmetic per byte that occupancy
    // matters more than deep unrolling (registers); plain adds unroll.
    constexpr int kThreads = 256, kUnroll = OP == tbk::kAdd ? 4 : 1;
    constexpr bool bin = tbk::ew_binary<OP>();
    const T* ap = static_cast<const T*>(a);
    const T* bp = static_cast<const T*>(b);
    T* op = static_cast<T*>(out);
    const bool vec_ok = tbh::aligned16(a) && (!bin || tbh::aligned16(b)) && tbh::aligned16(out);
    if (vec_ok) {
        const int64_t nvec = n / V;
        if (nvec > 0) {
            const int grid = tbh::ew_grid((nvec + kUnroll - 1) / kUnroll, kThreads, ds);
            k_ew<T, V, OP, kUnroll><<<grid, kThreads, 0, s>>>(ap, bp, op, nvec);
            TB_LAUNCH_CHECK("elementwise kernel");
        }
        const int64_t done = nvec * V, tail = n - done;
        if (tail > 0) {
            k_ew<T, 1, OP, 1><<<1, kThreads, 0, s>>>(ap + done, bin ? bp + done : nullptr, op + done,
                                                     tail);
            TB_LAUNCH_CHECK("elementwise tail kernel");
        }
        return TB_OK;
    }
    const int grid = tbh::ew_grid((n + kUnroll - 1) / kUnroll, kThreads, ds);
    k_ew<T, 1, OP, kUnroll><<<grid, kThreads, 0, s>>>(ap, bp, op, n);
    TB_LAUNCH_CHECK("elementwise kernel");
    return TB_OK;
}

template <int OP>
int run(int dtype, int64_t n, const void* a, const void* b, void* out, void* stream) {
    if (n < 0) return TB_ERR_INVALID_SHAPE;
    if (n == 0) return TB_OK;
    if (!a || !out || (tbk::ew_binary<OP>() && !b)) return TB_ERR_INVALID_ARG;
    cudaStream_t s = tbh::stream_of(stream);
    if (dtype == TB_DTYPE_F32) return launch<float, OP>(a, b, out, n, s);
    if (dtype == TB_DTYPE_BF16) return launch<__nv_bfloat16, OP>(a, b, out, n, s);
    return TB_ERR_UNSUPPORTED_DTYPE;
}

}  // namespace

extern "C" int tb_b200_silu(int dtype, int64_t n, const void* x, void* y, void* stream) {
    return run<tbk::kSilu>(dtype, n, x, nullptr, y, stream);
}

extern "C" int tb_b200_gelu(int dtype, int64_t n, const void* x, void* y, void* stream) {
    return run<tbk::kGelu>(dtype, n, x, nullptr, y, stream);
}

extern "C" int tb_b200_swiglu(int dtype, int64_t n, const void* gate, const void* up, void* out,
                              void* stream) {
    return run<tbk::kSwiglu>(dtype, n, gate, up, out, stream);
}

extern "C" int tb_b200_residual_add(int dtype, int64_t n, const void* x, const void* residual,
                                    void* y, void* stream) {
    return run<tbk::kAdd>(dtype, n, x, residual, y, stream);
}
