// k_chain.cu -- a transformer layer's three row-op groups in ONE launch.
//
// TransformerRunner::forward (include/tensorbit/run/ops.hpp:120-248) runs,
// per layer, RMSNorm (with the residual add), RoPE on Q/K, and SiLU(gate)*up.
// At decode batch sizes each of those is a few MB -- microseconds of HBM
// time, comparable to a kernel launch -- so the three are fused
// horizontally: the grid is split into block ranges, one per group, and each
// block runs the same body the standalone kernel runs (bodies.cuh), so the
// results are bit-identical to tb_b200_residual_rms_norm + tb_b200_rope_rows
// + tb_b200_swiglu.  The groups touch disjoint tensors, so their blocks run
// concurrently and the launch costs one launch latency instead of three;
// captured in a CUDA graph over the layers, a decode step is one graph
// launch.
//
// The fused path needs 16-byte-aligned rows; other shapes run the three
// standalone kernels back to back (same results).
//
// Launches use programmatic dependent launch: a chain kernel may be
// scheduled while the kernel before it in the stream drains its last wave.
// Each CTA first waits (griddepcontrol.wait) until that kernel has
// completed and its memory is visible, so nothing is read or written early;
// it then lets the next kernel's launch begin (launch_dependents), which
// happens once every CTA of this grid has started.  Over the 32 layers of a
// decode step the launch latency of layer l + 1 overlaps the tail of
// layer l.
#include <string.h>

#include "bodies.cuh"
#include "tb_internal.h"

namespace {

using tbk::Elt;

template <typename T>
struct ChainArgs {
    // residual + RMSNorm
    const T* x;
    const T* res;
    const T* w;
    T* h;
    T* y;
    int64_t rows;
    int hidden;
    float eps;
    int G;
    int64_t norm_blocks;
    // RoPE
    T* q;
    T* k;
    const int32_t* pos;
    int hq, hkv, d;
    const float2* table;
    int table_pos;
    int64_t rope_blocks;
    // SwiGLU
    const T* gate;
    const T* up;
    T* act;
    int64_t nvec;
    int64_t ew_blocks;
    tbk::RopeConst rc;
};

constexpr int kThreads = 256;

template <typename T, int ITEMS>
__global__ void __launch_bounds__(kThreads) k_chain(const __grid_constant__ ChainArgs<T> a) {
    constexpr int V = Elt<T>::kVec;
    __shared__ float red[32];
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    int64_t b = blockIdx.x;
    if (b < a.norm_blocks) {
        tbk::res_rms_body<T, V, ITEMS>(a.x, a.res, a.w, a.h, a.y, a.rows, a.hidden, a.eps, a.G, b,
                                       red);
        return;
    }
    b -= a.norm_blocks;
    if (b < a.rope_blocks) {
        tbk::rope_body<T, V, tbk::kRopePerRow, 4>(a.q, a.k, a.pos, a.hq, a.hkv, a.d, a.table,
                                                  a.table_pos, a.rc, b);
        return;
    }
    b -= a.rope_blocks;
    tbk::ew_body<T, V, tbk::kSwiglu, 1>(a.gate, a.up, a.act, a.nvec, b, a.ew_blocks);
}

template <typename T>
int launch_fused(const TbB200LayerChain* c, const tbh::DeviceState* ds, cudaStream_t s) {
    constexpr int V = Elt<T>::kVec;
    ChainArgs<T> a;
    memset(&a, 0, sizeof a);
    int items = 1;
    if (c->hidden > 0) {
        const tbh::NormCfg nc = tbh::norm_cfg(c->hidden / V, kThreads);
        items = nc.items;
        a.x = static_cast<const T*>(c->x);
        a.res = static_cast<const T*>(c->residual);
        a.w = static_cast<const T*>(c->norm_weight);
        a.h = static_cast<T*>(c->h_out);
        a.y = static_cast<T*>(c->y);
        a.rows = c->rows;
        a.hidden = (int)c->hidden;
        a.eps = c->eps;
        a.G = nc.G;
        const int per = kThreads / nc.G;
        a.norm_blocks = (c->rows + per - 1) / per;
    }
    if (c->n_q_heads + c->n_kv_heads > 0 && c->head_dim >= 2) {
        a.q = static_cast<T*>(c->q);
        a.k = static_cast<T*>(c->k);
        a.pos = c->positions;
        a.hq = c->n_q_heads;
        a.hkv = c->n_kv_heads;
        a.d = c->head_dim;
        a.table = reinterpret_cast<const float2*>(c->rope_table);
        a.table_pos = c->rope_table_positions;
        a.rope_blocks = c->rows;
        tbh::rope_inv_freq(c->theta, c->head_dim, a.rc.inv_freq);
    }
    if (c->intermediate > 0) {
        a.gate = static_cast<const T*>(c->gate);
        a.up = static_cast<const T*>(c->up);
        a.act = static_cast<T*>(c->act_out);
        a.nvec = c->rows * c->intermediate / V;
        a.ew_blocks = tbh::ew_grid(a.nvec, kThreads, ds);
    }
    const int64_t grid = a.norm_blocks + a.rope_blocks + a.ew_blocks;
    if (grid == 0) return TB_OK;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    switch (items) {
        case 1: e = cudaLaunchKernelEx(&cfg, k_chain<T, 1>, a); break;
        case 2: e = cudaLaunchKernelEx(&cfg, k_chain<T, 2>, a); break;
        default: e = cudaLaunchKernelEx(&cfg, k_chain<T, 4>, a); break;
    }
    if (e != cudaSuccess) {
        tbh::count_launch();
        tbh::set_error("layer chain kernel", e);
        return TB_ERR_DEVICE;
    }
    TB_LAUNCH_CHECK("layer chain kernel");
    return TB_OK;
}

bool fusable(const TbB200LayerChain* c, int vec) {
    using tbh::aligned16;
    if (c->hidden > 0) {
        if (c->hidden % vec || !aligned16(c->x) || !aligned16(c->y)) return false;
        if ((c->residual && !aligned16(c->residual)) || (c->norm_weight && !aligned16(c->norm_weight)) ||
            (c->h_out && !aligned16(c->h_out)))
            return false;
        if (tbh::norm_cfg(c->hidden / vec, kThreads).items == 0) return false;
    }
    if (c->n_q_heads + c->n_kv_heads > 0 && c->head_dim >= 2) {
        if (c->head_dim % vec || (c->n_q_heads && !aligned16(c->q)) ||
            (c->n_kv_heads && !aligned16(c->k)) || (c->rope_table && !aligned16(c->rope_table)))
            return false;
        if (c->head_dim / vec > kThreads) return false;
    }
    if (c->intermediate > 0) {
        if ((c->rows * c->intermediate) % vec || !aligned16(c->gate) || !aligned16(c->up) ||
            !aligned16(c->act_out))
            return false;
    }
    return true;
}

}  // namespace

extern "C" int tb_b200_layer_chain(const TbB200LayerChain* c, void* stream) {
    if (!c) return TB_ERR_INVALID_ARG;
    if (c->rows < 0 || c->hidden < 0 || c->intermediate < 0 || c->n_q_heads < 0 ||
        c->n_kv_heads < 0 || c->head_dim < 0 || c->rows > INT32_MAX || c->hidden > INT32_MAX)
        return TB_ERR_INVALID_SHAPE;
    if (c->dtype != TB_DTYPE_F32 && c->dtype != TB_DTYPE_BF16) return TB_ERR_UNSUPPORTED_DTYPE;
    if (c->head_dim / 2 > tbk::kRopeMaxPairs) return TB_ERR_INVALID_SHAPE;
    if (c->rows == 0) return TB_OK;
    const bool has_norm = c->hidden > 0;
    const bool has_rope = c->n_q_heads + c->n_kv_heads > 0 && c->head_dim >= 2;
    const bool has_act = c->intermediate > 0;
    if ((has_norm && (!c->x || !c->y)) ||
        (has_rope && ((c->n_q_heads && !c->q) || (c->n_kv_heads && !c->k) || !c->positions)) ||
        (has_act && (!c->gate || !c->up || !c->act_out)))
        return TB_ERR_INVALID_ARG;
    tbh::DeviceState* ds = tbh::current_device_state();
    if (!ds) return TB_ERR_DEVICE;
    cudaStream_t s = tbh::stream_of(stream);
    const int vec = c->dtype == TB_DTYPE_F32 ? 4 : 8;
    if (fusable(c, vec)) {
        if (c->dtype == TB_DTYPE_F32) return launch_fused<float>(c, ds, s);
        return launch_fused<__nv_bfloat16>(c, ds, s);
    }
    int rc = TB_OK;
    if (has_norm)
        rc = tb_b200_residual_rms_norm(c->dtype, c->rows, c->hidden, c->x, c->residual,
                                       c->norm_weight, c->h_out, c->y, c->eps, s);
    if (rc == TB_OK && has_rope)
        rc = tb_b200_rope_rows(c->dtype, c->rows, c->n_q_heads, c->n_kv_heads, c->head_dim, c->q,
                               c->k, c->positions, c->theta, c->rope_table,
                               c->rope_table_positions, s);
    if (rc == TB_OK && has_act)
        rc = tb_b200_swiglu(c->dtype, c->rows * c->intermediate, c->gate, c->up, c->act_out, s);
    return rc;
}
