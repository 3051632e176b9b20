// pin_registry.cpp -- the engine's C++ backend registry, compiled as the
// engine would compile it with the b200 backend, for checking the drop-in
// boundary on the CPU.
//
// TEST INFRASTRUCTURE ONLY.  Built by oracle/Makefile into oracle/_ref/:
//   * include/tensorbit/run/backend.hpp (tensorbit::run::BackendRegistry and
//     the op wrappers, backend.hpp:19-53 and on) is the reference's header,
//     unmodified;
//   * its "tensorbit/run/backend.h" resolves to a two-line stand-in that
//     includes this repository's include/tb_backend.h -- the header swap the
//     integration makes;
//   * -DTB_HAS_CUDA -Dtb_backend_cuda_init=tb_backend_b200_init binds the
//     reference's accelerator branch of BackendRegistry::init
//     (backend.hpp:27-35) to the b200 backend's init, i.e. the one-line
//     change the integration makes there;
//   * the reference's CPU kernels and adapters (src/ops/*.c,
//     src/backend/cpu/*.c without registry.c, whose registry half this
//     library provides) are linked in, and tb_backend_cpu_init below
//     registers them as src/backend/cpu/registry.c:63-84 does;
//   * the registry itself is libtb_b200.so's.
#include <cstring>

#include "tensorbit/run/backend.hpp"

extern "C" {

// The reference's CPU adapters (src/backend/cpu/*.c); the reference declares
// them inside src/backend/cpu/registry.c:7-20.
int tb_cpu_sparse_linear_dispatch(void*, const void**, int, const void*);
int tb_cpu_dense_linear_dispatch(void*, const void**, int, const void*);
int tb_cpu_rms_norm_dispatch(void*, const void**, int, const void*);
int tb_cpu_layer_norm_dispatch(void*, const void**, int, const void*);
int tb_cpu_gelu_dispatch(void*, const void**, int, const void*);
int tb_cpu_silu_dispatch(void*, const void**, int, const void*);
int tb_cpu_softmax_dispatch(void*, const void**, int, const void*);
int tb_cpu_attention_qkv_dispatch(void*, const void**, int, const void*);
int tb_cpu_scaled_dot_product_dispatch(void*, const void**, int, const void*);
int tb_cpu_rope_dispatch(void*, const void**, int, const void*);
int tb_cpu_residual_add_dispatch(void*, const void**, int, const void*);
int tb_cpu_embedding_dispatch(void*, const void**, int, const void*);
int tb_cpu_conv2d_dispatch(void*, const void**, int, const void*);
// The engine-side slots of the added ops (tensorbit-run_b200/engine/cpu_rowops.c).
void tb_cpu_rowops_fill(TbBackend* cpu);

int tb_backend_cpu_init(void) {
    TbBackend cpu;
    std::memset(&cpu, 0, sizeof cpu);
    cpu.name = "cpu";
    cpu.priority = 0;
    cpu.ops[TB_OP_SPARSE_LINEAR] = tb_cpu_sparse_linear_dispatch;
    cpu.ops[TB_OP_DENSE_LINEAR] = tb_cpu_dense_linear_dispatch;
    cpu.ops[TB_OP_RMS_NORM] = tb_cpu_rms_norm_dispatch;
    cpu.ops[TB_OP_LAYER_NORM] = tb_cpu_layer_norm_dispatch;
    cpu.ops[TB_OP_GELU] = tb_cpu_gelu_dispatch;
    cpu.ops[TB_OP_SILU] = tb_cpu_silu_dispatch;
    cpu.ops[TB_OP_SOFTMAX] = tb_cpu_softmax_dispatch;
    cpu.ops[TB_OP_ATTENTION_QKV] = tb_cpu_attention_qkv_dispatch;
    cpu.ops[TB_OP_SCALED_DOT_PRODUCT] = tb_cpu_scaled_dot_product_dispatch;
    cpu.ops[TB_OP_ROPE] = tb_cpu_rope_dispatch;
    cpu.ops[TB_OP_RESIDUAL_ADD] = tb_cpu_residual_add_dispatch;
    cpu.ops[TB_OP_EMBEDDING] = tb_cpu_embedding_dispatch;
    cpu.ops[TB_OP_CONV2D] = tb_cpu_conv2d_dispatch;
    tb_cpu_rowops_fill(&cpu);
    return tb_backend_register(&cpu);
}

// BackendRegistry::instance().init(); returns the registered count.
int pin_registry_init(void) {
    tensorbit::run::BackendRegistry::instance().init();
    return tensorbit::run::BackendRegistry::instance().count();
}

int pin_registry_has(const char* name) {
    return tensorbit::run::BackendRegistry::instance().has_backend(name) ? 1 : 0;
}

// Name of the backend tb_backend_get_best_device picks, or NULL.
const char* pin_registry_best(int op, int device) {
    const TbBackend* b = tb_backend_get_best_device((TbOpType)op, (TbDevice)device);
    return b ? b->name : nullptr;
}

// The reference's C++ wrapper rms_norm(Tensor&, ...) (backend.hpp) on host
// tensors: it must reach the CPU adapters.
int pin_registry_rms_norm_host(float* y, const float* x, const float* w, size_t n, float eps) {
    using namespace tensorbit::run;
    Tensor ty = Tensor::wrap(y, {n}, Dtype::kF32, DeviceLocation::kHost);
    Tensor tx = Tensor::wrap(const_cast<float*>(x), {n}, Dtype::kF32, DeviceLocation::kHost);
    Tensor tw = Tensor::wrap(const_cast<float*>(w), {n}, Dtype::kF32, DeviceLocation::kHost);
    return rms_norm(ty, tx, tw, eps);
}

// The added ops through tb_dispatch_* on host f32 tensors of [rows, cols]:
// they must reach the CPU backend's composition slots.
static TbTensor host2(void* p, size_t rows, size_t cols, TbDtype dt = TB_DTYPE_F32) {
    TbTensor t;
    std::memset(&t, 0, sizeof t);
    t.data = p;
    t.rank = 2;
    t.shape[0] = rows;
    t.shape[1] = cols;
    t.dtype = dt;
    t.device = TB_DEVICE_CPU;
    return t;
}
static TbTensor host3(void* p, size_t a, size_t b, size_t c) {
    TbTensor t = host2(p, a, b);
    t.rank = 3;
    t.shape[2] = c;
    return t;
}

int pin_registry_residual_rms_norm_host(float* y, float* h, const float* x, const float* r,
                                        const float* w, size_t rows, size_t cols, float eps) {
    TbTensor ty = host2(y, rows, cols), th = host2(h, rows, cols);
    TbTensor tx = host2(const_cast<float*>(x), rows, cols);
    TbTensor tr = host2(const_cast<float*>(r), rows, cols);
    TbTensor tw = host2(const_cast<float*>(w), 1, cols);
    tw.rank = 1;
    tw.shape[0] = cols;
    return tb_dispatch_residual_rms_norm(&ty, &th, &tx, &tr, &tw, eps);
}

int pin_registry_swiglu_host(float* out, const float* g, const float* u, size_t rows, size_t cols) {
    TbTensor to = host2(out, rows, cols), tg = host2(const_cast<float*>(g), rows, cols);
    TbTensor tu = host2(const_cast<float*>(u), rows, cols);
    return tb_dispatch_swiglu(&to, &tg, &tu);
}

int pin_registry_argmax_host(int32_t* out, const float* x, size_t rows, size_t cols) {
    TbTensor tx = host2(const_cast<float*>(x), rows, cols);
    TbTensor to = host2(out, rows, 1, TB_DTYPE_I32);
    to.rank = 1;
    to.shape[0] = rows;
    return tb_dispatch_argmax(&to, &tx);
}

int pin_registry_rope_rows_host(float* q, float* k, const int32_t* pos, size_t rows, size_t hq,
                                size_t hkv, size_t d, float theta) {
    TbTensor tq = host3(q, rows, hq, d), tk = host3(k, rows, hkv, d);
    return tb_dispatch_rope_rows(&tq, &tk, pos, theta, (int)d, 0);
}

int pin_registry_layer_chain_host(float* y, float* h, float* act, const float* x, const float* r,
                                  const float* w, float* q, float* k, const float* g,
                                  const float* u, const int32_t* pos, size_t rows, size_t hidden,
                                  size_t hq, size_t hkv, size_t d, size_t inter, float eps,
                                  float theta) {
    TbTensor ty = host2(y, rows, hidden), th = host2(h, rows, hidden);
    TbTensor ta = host2(act, rows, inter);
    TbTensor tx = host2(const_cast<float*>(x), rows, hidden);
    TbTensor tr = host2(const_cast<float*>(r), rows, hidden);
    TbTensor tw = host2(const_cast<float*>(w), 1, hidden);
    tw.rank = 1;
    tw.shape[0] = hidden;
    TbTensor tq = host3(q, rows, hq, d), tk = host3(k, rows, hkv, d);
    TbTensor tg = host2(const_cast<float*>(g), rows, inter);
    TbTensor tu = host2(const_cast<float*>(u), rows, inter);
    TbLayerChainParams p;
    p.eps = eps;
    p.positions = pos;
    p.theta = theta;
    p.head_dim = (int)d;
    p.max_position = 0;
    return tb_dispatch_layer_chain(&ty, &th, &ta, &tx, &tr, &tw, &tq, &tk, &tg, &tu, &p);
}

}  // extern "C"
