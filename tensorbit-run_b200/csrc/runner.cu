// runner.cu -- the engine's single-token decoder forward on the device
// (tensorbit::run::TransformerRunner, include/tensorbit/run/ops.hpp:33-288).
//
// Per token, on the runner's own stream (ops.hpp line numbers):
//   embedding gather of the token from the device copy of its id      :92
//   per layer whose q/k/v exist (:109):
//     x = rms_norm(x) * input_norm, in place                           :119
//     q, k, v = W x (2:4 sparse GEMV over the mask, or dense)          :140-149
//     RoPE of q and k at the device position (host-built table)        :159
//     decode attention: append k/v to the cache, attend (one launch)   :162-204
//     x = x + Wo attn (the GEMV's epilogue adds the residual)          :207-218
//     x_mlp = rms_norm(x) * post_norm                                  :221-223
//     g = silu(Wg x_mlp) * (Wu x_mlp); x = x + Wd g                    :226-256
//   x = rms_norm(x) * final_norm; logits = Wlm x                       :260-281
//   position += 1 on the device                                        :284
// The position and the token id live in device memory, so the whole step
// is captured once as a CUDA graph and replayed for every token
// (use_graph); eager launches otherwise.  Weights stay resident: f32 device
// tensors are borrowed, host tensors copied once, INT4/INT8 tensors
// dequantised once with tb_b200_dequant (the reference dequantises on every
// use, to the same values).
#include <cmath>
#include <cstring>
#include <initializer_list>
#include <new>
#include <vector>

#include "gemv.cuh"
#include "tb_internal.h"

#include "runner_kernels.h"

namespace {

__global__ void k_advance(int32_t* pos) { *pos += 1; }

struct Proj {
    const float* w = nullptr;    // f32 weights (INT8/INT4: the quantized bytes)
    const uint8_t* mask = nullptr;
    const void* vals = nullptr;  // packed 2:4 form, when the mask allows it
    const uint8_t* idx = nullptr;
    int64_t rows = 0, cols = 0;
    int qbits = 0;               // 8 or 4: kept quantized, expanded inside the GEMV
    const float* qscales = nullptr;
    int64_t nsc = 0;
    int gshift = 31;             // log2(group size), 31 for one group
};

struct Layer {
    Proj q, k, v, o, gate, up, down;
    const float* in_norm = nullptr;
    const float* post_norm = nullptr;
};

struct Runner {
    TbB200RunnerDesc cfg{};
    int device = 0;
    cudaStream_t stream = nullptr;
    std::vector<void*> owned;  // device allocations
    const float* embed = nullptr;
    const float* final_norm = nullptr;
    const float* lm_head = nullptr;
    std::vector<Layer> layers;
    float *x = nullptr, *xn = nullptr, *q = nullptr, *k = nullptr, *v = nullptr,
          *attn = nullptr;
    float *xm = nullptr, *g = nullptr, *u = nullptr, *logits = nullptr;
    float *kc = nullptr, *vc = nullptr, *rope = nullptr;
    int32_t* dstate = nullptr;  // [0] position, [1] token
    int att_splits = 1;         // CTAs per attention row when rows are long
    float* att_part = nullptr;  // their partial results
    int* att_count = nullptr;   // their per-row arrival counters
    int* flag = nullptr;        // packing verdict of one layer
    int pos = 0;
    int launches = 0;
    cudaGraphExec_t exec = nullptr;
    cudaGraph_t graph = nullptr;
};

int dev_alloc(Runner* r, size_t bytes, void** p) {
    TB_CUDA_TRY(cudaMalloc(p, bytes ? bytes : 16));
    r->owned.push_back(*p);
    return TB_OK;
}

// An f32 device copy of a weight tensor (borrowed when it already is one).
int materialize(Runner* r, const TbB200Weight& w, const float** out) {
    *out = nullptr;
    if (!w.data) return TB_OK;
    if (w.rows <= 0 || w.cols < 0) return TB_ERR_INVALID_SHAPE;
    const int64_t n = w.cols ? w.rows * w.cols : w.rows;
    int on_dev = 0;
    tb_b200_is_device_ptr(w.data, &on_dev);
    if (w.dtype == TB_DTYPE_F32) {
        if (on_dev) {
            *out = static_cast<const float*>(w.data);
            return TB_OK;
        }
        void* d = nullptr;
        int rc = dev_alloc(r, (size_t)n * 4, &d);
        if (rc) return rc;
        TB_CUDA_TRY(cudaMemcpyAsync(d, w.data, (size_t)n * 4, cudaMemcpyHostToDevice, r->stream));
        *out = static_cast<const float*>(d);
        return TB_OK;
    }
    if (w.dtype != TB_DTYPE_INT4 && w.dtype != TB_DTYPE_INT8) return TB_ERR_UNSUPPORTED_DTYPE;
    const size_t qbytes = w.dtype == TB_DTYPE_INT4 ? (size_t)(n + 1) / 2 : (size_t)n;
    const void* src = w.data;
    const float* sc = w.scales;
    if (!on_dev) {
        void* d = nullptr;
        int rc = dev_alloc(r, qbytes, &d);
        if (rc) return rc;
        TB_CUDA_TRY(cudaMemcpyAsync(d, w.data, qbytes, cudaMemcpyHostToDevice, r->stream));
        src = d;
    }
    int sc_dev = 0;
    tb_b200_is_device_ptr(w.scales, &sc_dev);
    if (w.n_scales > 0 && w.scales && !sc_dev) {
        void* d = nullptr;
        int rc = dev_alloc(r, (size_t)w.n_scales * 4, &d);
        if (rc) return rc;
        TB_CUDA_TRY(cudaMemcpyAsync(d, w.scales, (size_t)w.n_scales * 4, cudaMemcpyHostToDevice,
                                    r->stream));
        sc = static_cast<const float*>(d);
    }
    void* d = nullptr;
    int rc = dev_alloc(r, (size_t)n * 4, &d);
    if (rc) return rc;
    rc = tb_b200_dequant(w.dtype, n, src, sc, w.n_scales, w.group_size, TB_DTYPE_F32, d, r->stream);
    if (rc) return rc;
    *out = static_cast<const float*>(d);
    return TB_OK;
}

int materialize_vec(Runner* r, const float* p, int64_t n, const float** out) {
    TbB200Weight w{};
    w.data = p;
    w.dtype = TB_DTYPE_F32;
    w.rows = n;
    w.cols = 0;
    return materialize(r, w, out);
}

int materialize_mask(Runner* r, const TbB200Weight& w, const uint8_t** out) {
    *out = nullptr;
    if (!w.data || !w.mask) return TB_OK;
    int on_dev = 0;
    tb_b200_is_device_ptr(w.mask, &on_dev);
    if (on_dev) {
        *out = w.mask;
        return TB_OK;
    }
    const size_t bytes = (size_t)w.rows * (size_t)(w.cols / 4);
    void* d = nullptr;
    int rc = dev_alloc(r, bytes, &d);
    if (rc) return rc;
    TB_CUDA_TRY(cudaMemcpyAsync(d, w.mask, bytes, cudaMemcpyHostToDevice, r->stream));
    *out = static_cast<const uint8_t*>(d);
    return TB_OK;
}

void free_owned(Runner* r, const void* p) {
    for (size_t i = 0; i < r->owned.size(); ++i)
        if (r->owned[i] == p) {
            cudaFree(r->owned[i]);
            r->owned.erase(r->owned.begin() + (long)i);
            return;
        }
}

// Packed 2:4 form of a masked projection, when every group keeps at most
// two weights and the groups pair up.
int pack(Runner* r, Proj* p) {
    const int64_t groups = p->cols / 4;
    if (!p->mask || groups == 0 || groups % 2) return TB_OK;
    const int64_t pairs = groups / 2;
    void *vals = nullptr, *idx = nullptr;
    int rc;
    if ((rc = dev_alloc(r, (size_t)(p->rows * pairs) * 16, &vals))) return rc;
    if ((rc = dev_alloc(r, (size_t)(p->rows * tbk::packed_idx_stride(pairs)), &idx))) return rc;
    TB_CUDA_TRY(cudaMemsetAsync(r->flag, 0, sizeof(int), r->stream));
    if ((rc = tb_b200_sparse24_pack(p->rows, p->cols, p->w, p->mask, vals, (uint8_t*)idx, r->flag,
                                    r->stream)))
        return rc;
    int bad = 0;
    TB_CUDA_TRY(cudaMemcpyAsync(&bad, r->flag, sizeof(int), cudaMemcpyDeviceToHost, r->stream));
    TB_CUDA_TRY(cudaStreamSynchronize(r->stream));
    if (bad) {  // three or four weights kept in some group: dense-with-mask
        free_owned(r, vals);
        free_owned(r, idx);
        return TB_OK;
    }
    p->vals = vals;
    p->idx = static_cast<const uint8_t*>(idx);
    free_owned(r, p->w);    // uploaded dense copies are no longer needed
    free_owned(r, p->mask);
    p->w = static_cast<const float*>(vals);  // non-null: the projection exists
    p->mask = nullptr;
    return TB_OK;
}

// A device copy of `bytes` at p (borrowed when p already is device memory).
int upload(Runner* r, const void* p, size_t bytes, const void** out) {
    int on_dev = 0;
    tb_b200_is_device_ptr(p, &on_dev);
    if (on_dev) {
        *out = p;
        return TB_OK;
    }
    void* d = nullptr;
    int rc = dev_alloc(r, bytes, &d);
    if (rc) return rc;
    TB_CUDA_TRY(cudaMemcpyAsync(d, p, bytes, cudaMemcpyHostToDevice, r->stream));
    *out = d;
    return TB_OK;
}

// An unmasked INT8/INT4 projection whose rows are whole words of 32 inputs
// and whose scale groups are 0 (one group) or a power of two of at least 8
// stays quantized: the fused GEMV expands each weight to the same
// (float)q * scale that Model::get_weight_fp32 gives.
int keep_quantized(Runner* r, const TbB200Weight& w, Proj* p) {
    const int64_t gs = (int64_t)w.group_size;
    const int64_t n = w.rows * w.cols;
    const size_t qbytes = w.dtype == TB_DTYPE_INT4 ? (size_t)(n + 1) / 2 : (size_t)n;
    const void *q = nullptr, *sc = nullptr;
    int rc = upload(r, w.data, qbytes, &q);
    if (rc) return rc;
    if (!tbh::aligned16(q)) return TB_ERR_INVALID_ARG;  // caller falls back
    if (w.n_scales > 0 && w.scales) {
        if ((rc = upload(r, w.scales, (size_t)w.n_scales * 4, &sc))) return rc;
    }
    p->w = static_cast<const float*>(q);
    p->qbits = w.dtype == TB_DTYPE_INT4 ? 4 : 8;
    p->qscales = static_cast<const float*>(sc);
    p->nsc = sc ? w.n_scales : 0;
    p->gshift = 31;  // one group
    if (gs > 0 && gs < n)
        for (p->gshift = 0; ((int64_t)1 << p->gshift) < gs; ++p->gshift) {
        }
    return TB_OK;
}

bool quantized_fits(const TbB200Weight& w) {
    if ((w.dtype != TB_DTYPE_INT8 && w.dtype != TB_DTYPE_INT4) || w.mask) return false;
    const int64_t gs = (int64_t)w.group_size;
    const int64_t n = w.rows * w.cols;
    const int64_t groups = gs == 0 || gs >= n ? 1 : (n + gs - 1) / gs;
    // every group has its scale (the kernel reads one per group, unchecked)
    return w.cols % 32 == 0 && n < ((int64_t)1 << 31) && w.scales && w.n_scales >= groups &&
           (gs == 0 || (gs >= 8 && (gs & (gs - 1)) == 0));
}

int make_proj(Runner* r, const TbB200Weight& w, int64_t rows, int64_t cols, Proj* p) {
    *p = Proj{};
    if (!w.data) return TB_OK;
    if (w.rows != rows || w.cols != cols) return TB_ERR_INVALID_SHAPE;
    p->rows = rows;
    p->cols = cols;
    if (quantized_fits(w)) {
        const int rq = keep_quantized(r, w, p);
        if (rq == TB_OK) return TB_OK;
        if (rq != TB_ERR_INVALID_ARG) return rq;
        *p = Proj{};  // an unaligned borrowed tensor: dequantise it below
        p->rows = rows;
        p->cols = cols;
    }
    int rc = materialize(r, w, &p->w);
    if (rc) return rc;
    rc = materialize_mask(r, w, &p->mask);
    if (rc) return rc;
    p->rows = rows;
    p->cols = cols;
    return pack(r, p);
}

int fused_layout(const Proj& p);
tbh::GemvSeg seg_of(const Proj& p, float* y);
struct Norm;
int fused_one(Runner* r, int layout, const Proj& p, const float* x, const float* res, float* y);

// y = W x, plus `res` (which may be y itself) when given.
int project(Runner* r, const Proj& p, const float* x, const float* res, float* y) {
    if (p.qbits) return fused_one(r, fused_layout(p), p, x, res, y);  // only the fused GEMV reads it
    r->launches++;
    if (p.vals)
        return tb_b200_sparse24_linear(p.rows, p.cols, x, p.vals, p.idx, res, y, r->stream);
    if (p.mask)  // the runner's projections run as 2:4 groups (registry.c:93)
        return tb_b200_sparse_linear(p.rows, p.cols, x, p.w, p.mask, res, y, 2, 4, r->stream);
    return tb_b200_dense_linear(p.rows, p.cols, x, p.w, res, y, r->stream);
}

// The fused-GEMV layout a projection can take (k_runner.cu), or -1.
int fused_layout(const Proj& p) {
    if (!p.w) return -1;
    if (p.qbits) return p.qbits == 8 ? tbh::kInt8 : tbh::kInt4;
    if (p.vals) return p.cols % 8 == 0 ? tbh::kPacked : -1;
    if (p.mask) return -1;  // dense-with-mask: the library's sparse GEMV
    return p.cols % 4 == 0 && tbh::aligned16(p.w) ? tbh::kDense : -1;
}

int common_layout(const Proj& a, const Proj& b, const Proj* c = nullptr) {
    const int l = fused_layout(a);
    if (l < 0 || fused_layout(b) != l || (c && fused_layout(*c) != l)) return -1;
    return l;
}

tbh::GemvSeg seg_of(const Proj& p, float* y) {
    tbh::GemvSeg g;
    g.w = p.vals ? p.vals : p.w;
    g.idx = p.idx;
    g.y = y;
    g.rows = p.rows;
    g.scales = p.qscales;
    g.n_scales = p.nsc;
    g.gshift = p.gshift;
    return g;
}

// One fused GEMV over 1-3 projections sharing the input x.
struct Norm {  // the RMSNorm a fused GEMV applies to its input first
    bool on = false;
    const float* w = nullptr;
    float* out = nullptr;
};

int fused(Runner* r, int layout, int epi, std::initializer_list<tbh::GemvSeg> segs,
          const float* x, int64_t cols, const float* res = nullptr, float* act = nullptr,
          Norm norm = Norm{}, int32_t* advance = nullptr) {
    const TbB200RunnerDesc& c = r->cfg;
    tbh::GemvArgs a{};
    int n = 0;
    for (const tbh::GemvSeg& g : segs) a.seg[n++] = g;
    a.nseg = n;
    a.cols = cols;
    a.x = x;
    a.res = res;
    a.norm = norm.on ? 1 : 0;
    a.norm_w = norm.w;
    a.eps = c.norm_eps;
    a.norm_out = norm.out;
    a.act = act;
    a.rope = reinterpret_cast<const float2*>(r->rope);
    a.rope_positions = c.max_seq;
    a.pos = r->dstate;
    a.head_dim = c.head_dim;
    a.rope_segs = 2;
    a.advance = advance;
    const tbh::DeviceState* ds = tbh::current_device_state();
    a.status = ds ? ds->status : nullptr;
    r->launches++;
    return tbh::fused_gemv(a, layout, epi, r->stream);
}

// A single projection through the fused GEMV (plain, or with the residual).
int fused_one(Runner* r, int layout, const Proj& p, const float* x, const float* res, float* y) {
    return fused(r, layout, res ? tbh::kResidual : tbh::kPlain, {seg_of(p, y)}, x, p.cols, res);
}

// The token's decoder step, queued on the runner's stream: 5 launches per
// layer when every projection group shares a fused layout (the norms run as
// the prologue of the GEMV that consumes them).
int enqueue(Runner* r) {
    const TbB200RunnerDesc& c = r->cfg;
    const int H = c.hidden;
    cudaStream_t s = r->stream;
    int rc;
    r->launches = 0;
#define TRY(call)                              \
    do {                                       \
        if ((rc = (call)) != TB_OK) return rc; \
    } while (0)
    TRY(tb_b200_embedding(TB_DTYPE_F32, 1, H, c.vocab, r->dstate + 1, r->embed, r->x, s));
    r->launches++;
    for (const Layer& L : r->layers) {
        if (!L.q.w || !L.k.w || !L.v.w) continue;  // ops.hpp:109
        // x = rms_norm(x) * input_norm (ops.hpp:119), then q, k, v and RoPE
        const float* xn;  // where the normalised x (the new residual stream) is
        const int lqkv = common_layout(L.q, L.k, &L.v);
        if (lqkv >= 0) {
            Norm nm;
            nm.on = true;
            nm.w = L.in_norm;
            nm.out = r->xn;
            TRY(fused(r, lqkv, tbh::kRope,
                      {seg_of(L.q, r->q), seg_of(L.k, r->k), seg_of(L.v, r->v)}, r->x, H,
                      nullptr, nullptr, nm));
            xn = r->xn;
        } else {
            TRY(tbh::runner_norm(H, r->x, L.in_norm, r->x, c.norm_eps, s));
            r->launches++;
            TRY(project(r, L.q, r->x, nullptr, r->q));
            TRY(project(r, L.k, r->x, nullptr, r->k));
            TRY(project(r, L.v, r->x, nullptr, r->v));
            TRY(tb_b200_rope_rows(TB_DTYPE_F32, 1, c.n_heads, c.n_kv_heads, c.head_dim, r->q, r->k,
                                  r->dstate, c.rope_theta, r->rope, c.max_seq, s));
            r->launches++;
            xn = r->x;
        }
        const size_t layer_off = (size_t)(&L - r->layers.data()) * (size_t)c.max_seq *
                                 (size_t)c.n_kv_heads * (size_t)c.head_dim;
        TRY(tbh::decode_attention_launch(c.attention, c.n_heads, c.n_kv_heads, c.head_dim,
                                         c.max_seq, r->dstate, r->q, r->k, r->v,
                                         r->kc + layer_off, r->vc + layer_off, r->attn, s, true,
                                         r->att_splits, r->att_part, r->att_count));
        r->launches++;
        if (L.o.w) {  // x = x_normalised + Wo attn (ops.hpp:207-218)
            const int lo = fused_layout(L.o);
            if (lo >= 0)
                TRY(fused(r, lo, tbh::kResidual, {seg_of(L.o, r->x)}, r->attn, L.o.cols, xn));
            else
                TRY(project(r, L.o, r->attn, xn, r->x));
        } else if (xn != r->x) {
            TB_CUDA_TRY(cudaMemcpyAsync(r->x, xn, (size_t)H * 4, cudaMemcpyDeviceToDevice, s));
        }
        if (L.gate.w && L.up.w && c.intermediate > 0) {  // ops.hpp:221-256
            const int lgu = common_layout(L.gate, L.up);
            if (lgu >= 0) {
                Norm nm;
                nm.on = true;
                nm.w = L.post_norm;
                TRY(fused(r, lgu, tbh::kSwiglu, {seg_of(L.gate, r->g), seg_of(L.up, r->u)}, r->x,
                          H, nullptr, r->g, nm));
            } else {
                TRY(tbh::runner_norm(H, r->x, L.post_norm, r->xm, c.norm_eps, s));
                r->launches++;
                TRY(project(r, L.gate, r->xm, nullptr, r->g));
                TRY(project(r, L.up, r->xm, nullptr, r->u));
                TRY(tb_b200_swiglu(TB_DTYPE_F32, c.intermediate, r->g, r->u, r->g, s));
                r->launches++;
            }
            if (L.down.w) {
                const int ld = fused_layout(L.down);
                if (ld >= 0)
                    TRY(fused(r, ld, tbh::kResidual, {seg_of(L.down, r->x)}, r->g, L.down.cols,
                              r->x));
                else
                    TRY(project(r, L.down, r->g, r->x, r->x));
            }
        }
    }
    // x = rms_norm(x) * final_norm; logits = Wlm x; position += 1 (ops.hpp:260-284)
    Proj lm;
    lm.w = r->lm_head;
    lm.rows = c.vocab;
    lm.cols = H;
    const int ll = fused_layout(lm);
    if (ll >= 0) {
        Norm nm;
        nm.on = true;
        nm.w = r->final_norm;
        TRY(fused(r, ll, tbh::kPlain, {seg_of(lm, r->logits)}, r->x, H, nullptr, nullptr, nm,
                  r->dstate));
    } else {
        TRY(tbh::runner_norm(H, r->x, r->final_norm, r->x, c.norm_eps, s));
        r->launches++;
        TRY(tb_b200_dense_linear(c.vocab, H, r->x, r->lm_head, nullptr, r->logits, s));
        r->launches++;
        k_advance<<<1, 1, 0, s>>>(r->dstate);
        TB_LAUNCH_CHECK("runner position kernel");
        r->launches++;
    }
#undef TRY
    return TB_OK;
}

void release(Runner* r) {
    if (!r) return;
    if (r->exec) cudaGraphExecDestroy(r->exec);
    if (r->graph) cudaGraphDestroy(r->graph);
    if (r->stream) cudaStreamSynchronize(r->stream);
    for (void* p : r->owned) cudaFree(p);
    if (r->stream) cudaStreamDestroy(r->stream);
    delete r;
}

int create(const TbB200RunnerDesc* d, Runner* r) {
    const TbB200RunnerDesc& c = *d;
    if (c.hidden <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 || c.head_dim <= 0 ||
        c.n_heads % c.n_kv_heads || c.vocab <= 0 || c.max_seq <= 0 || c.layers < 0 ||
        c.intermediate < 0 || c.head_dim % 2)
        return TB_ERR_INVALID_SHAPE;
    if (c.attention != TB_B200_ATTN_REFERENCE && c.attention != TB_B200_ATTN_STANDARD)
        return TB_ERR_INVALID_ARG;
    if (!c.embed.data || (c.layers > 0 && !c.layer)) return TB_ERR_INVALID_ARG;
    r->cfg = c;
    r->cfg.layer = nullptr;
    TB_CUDA_TRY(cudaGetDevice(&r->device));
    TB_CUDA_TRY(cudaStreamCreateWithFlags(&r->stream, cudaStreamNonBlocking));
    int rc = tbh::decode_attention_setup(c.head_dim, c.max_seq);
    if (rc) return rc;
    if ((rc = tbh::fused_gemv_setup(c.hidden))) return rc;
    const int64_t H = c.hidden, I = c.intermediate, V = c.vocab;
    const int64_t qd = (int64_t)c.n_heads * c.head_dim, kvd = (int64_t)c.n_kv_heads * c.head_dim;
    if (c.embed.rows != V || c.embed.cols != H) return TB_ERR_INVALID_SHAPE;
    if ((rc = materialize(r, c.embed, &r->embed))) return rc;
    if ((rc = materialize_vec(r, c.final_norm, H, &r->final_norm))) return rc;
    if (c.lm_head.data) {
        if (c.lm_head.rows != V || c.lm_head.cols != H) return TB_ERR_INVALID_SHAPE;
        if ((rc = materialize(r, c.lm_head, &r->lm_head))) return rc;
    } else {
        r->lm_head = r->embed;  // ops.hpp:269-273
    }
    void* fp = nullptr;
    if ((rc = dev_alloc(r, sizeof(int), &fp))) return rc;
    r->flag = static_cast<int*>(fp);
    r->layers.resize((size_t)c.layers);
    for (int l = 0; l < c.layers; l++) {
        const TbB200RunnerLayer& s = c.layer[l];
        Layer& L = r->layers[(size_t)l];
        if ((rc = make_proj(r, s.q, qd, H, &L.q)) || (rc = make_proj(r, s.k, kvd, H, &L.k)) ||
            (rc = make_proj(r, s.v, kvd, H, &L.v)) || (rc = make_proj(r, s.o, H, qd, &L.o)) ||
            (rc = make_proj(r, s.gate, I, H, &L.gate)) || (rc = make_proj(r, s.up, I, H, &L.up)) ||
            (rc = make_proj(r, s.down, H, I, &L.down)) ||
            (rc = materialize_vec(r, s.input_norm, H, &L.in_norm)) ||
            (rc = materialize_vec(r, s.post_norm, H, &L.post_norm)))
            return rc;
    }
    void* p;
    const size_t f = sizeof(float);
    if ((rc = dev_alloc(r, (size_t)H * f, &p))) return rc;
    r->x = (float*)p;
    if ((rc = dev_alloc(r, (size_t)H * f, &p))) return rc;
    r->xn = (float*)p;
    if ((rc = dev_alloc(r, (size_t)qd * f, &p))) return rc;
    r->q = (float*)p;
    if ((rc = dev_alloc(r, (size_t)kvd * f, &p))) return rc;
    r->k = (float*)p;
    if ((rc = dev_alloc(r, (size_t)kvd * f, &p))) return rc;
    r->v = (float*)p;
    if ((rc = dev_alloc(r, (size_t)qd * f, &p))) return rc;
    r->attn = (float*)p;
    if ((rc = dev_alloc(r, (size_t)H * f, &p))) return rc;
    r->xm = (float*)p;
    if ((rc = dev_alloc(r, (size_t)(I > 0 ? I : 1) * f, &p))) return rc;
    r->g = (float*)p;
    if ((rc = dev_alloc(r, (size_t)(I > 0 ? I : 1) * f, &p))) return rc;
    r->u = (float*)p;
    if ((rc = dev_alloc(r, (size_t)V * f, &p))) return rc;
    r->logits = (float*)p;
    const size_t cache = (size_t)(c.layers > 0 ? c.layers : 1) * (size_t)c.max_seq * (size_t)kvd * f;
    if ((rc = dev_alloc(r, cache, &p))) return rc;
    r->kc = (float*)p;
    if ((rc = dev_alloc(r, cache, &p))) return rc;
    r->vc = (float*)p;
    if ((rc = dev_alloc(r, (size_t)c.max_seq * c.head_dim * f, &p))) return rc;
    r->rope = (float*)p;
    if ((rc = tb_b200_rope_table(c.rope_theta, c.head_dim, c.max_seq, r->rope, r->stream)))
        return rc;
    if ((rc = dev_alloc(r, 2 * sizeof(int32_t), &p))) return rc;
    r->dstate = (int32_t*)p;
    r->att_splits = c.attention == TB_B200_ATTN_STANDARD
                        ? tbh::decode_attention_splits(c.n_heads, c.max_seq)
                        : 1;  // the reference's rows attend at most n_heads keys
    if (r->att_splits > 1) {
        // One partials buffer and one set of arrival counters serve every
        // layer's attention launch.  That is safe only while consecutive
        // attention launches are fully ordered: every kernel between two of
        // them (o-projection, gate/up, down, the next layer's QKV) executes
        // griddepcontrol.wait before its first memory access, so under
        // programmatic dependent launch a layer's attention cannot start
        // before the previous layer's has finished and reset its counters.
        // A kernel added to the step without that wait would let two
        // attention launches overlap on these buffers.
        if ((rc = dev_alloc(r, (size_t)c.n_heads * r->att_splits * (c.head_dim + 2) * f, &p)))
            return rc;
        r->att_part = (float*)p;
        if ((rc = dev_alloc(r, (size_t)c.n_heads * sizeof(int), &p))) return rc;
        r->att_count = (int*)p;
        TB_CUDA_TRY(cudaMemsetAsync(r->att_count, 0, (size_t)c.n_heads * sizeof(int), r->stream));
    }
    TB_CUDA_TRY(cudaMemsetAsync(r->dstate, 0, 2 * sizeof(int32_t), r->stream));
    TB_CUDA_TRY(cudaMemsetAsync(r->x, 0, (size_t)H * f, r->stream));
    TB_CUDA_TRY(cudaStreamSynchronize(r->stream));
    if (c.use_graph) {
        TB_CUDA_TRY(cudaStreamBeginCapture(r->stream, cudaStreamCaptureModeThreadLocal));
        rc = enqueue(r);
        cudaGraph_t graph = nullptr;
        const cudaError_t e = cudaStreamEndCapture(r->stream, &graph);
        if (rc) {
            if (graph) cudaGraphDestroy(graph);
            return rc;
        }
        if (e != cudaSuccess) {
            tbh::set_error("runner graph capture", e);
            return TB_ERR_DEVICE;
        }
        r->graph = graph;
        TB_CUDA_TRY(cudaGraphInstantiate(&r->exec, graph, 0));
    }
    return TB_OK;
}

}  // namespace

extern "C" int tb_b200_runner_create(const TbB200RunnerDesc* desc, void** runner) {
    if (!desc || !runner) return TB_ERR_INVALID_ARG;
    *runner = nullptr;
    Runner* r = new (std::nothrow) Runner();
    if (!r) return TB_ERR_OOM;
    const int rc = create(desc, r);
    if (rc != TB_OK) {
        release(r);
        return rc;
    }
    *runner = r;
    return TB_OK;
}

extern "C" int tb_b200_runner_forward(void* runner, int32_t token, const float** logits_dev) {
    Runner* r = static_cast<Runner*>(runner);
    if (!r) return TB_ERR_INVALID_ARG;
    if (token < 0 || token >= r->cfg.vocab) return TB_ERR_INVALID_ARG;
    if (r->pos >= r->cfg.max_seq) return TB_ERR_INVALID_SHAPE;
    // from pageable memory: the copy takes the value before it returns
    const int32_t tok = token;
    TB_CUDA_TRY(cudaMemcpyAsync(r->dstate + 1, &tok, sizeof(int32_t), cudaMemcpyHostToDevice,
                                r->stream));
    if (r->exec) {
        TB_CUDA_TRY(cudaGraphLaunch(r->exec, r->stream));
    } else {
        const int rc = enqueue(r);
        if (rc) return rc;
    }
    r->pos++;
    if (logits_dev) *logits_dev = r->logits;
    return TB_OK;
}

extern "C" int tb_b200_runner_logits(void* runner, float* logits_host) {
    Runner* r = static_cast<Runner*>(runner);
    if (!r || !logits_host) return TB_ERR_INVALID_ARG;
    TB_CUDA_TRY(cudaMemcpyAsync(logits_host, r->logits, (size_t)r->cfg.vocab * sizeof(float),
                                cudaMemcpyDeviceToHost, r->stream));
    TB_CUDA_TRY(cudaStreamSynchronize(r->stream));
    return TB_OK;
}

extern "C" int tb_b200_runner_reset(void* runner) {
    Runner* r = static_cast<Runner*>(runner);
    if (!r) return TB_ERR_INVALID_ARG;
    TB_CUDA_TRY(cudaMemsetAsync(r->dstate, 0, sizeof(int32_t), r->stream));
    r->pos = 0;
    return TB_OK;
}

extern "C" int tb_b200_runner_position(void* runner, int* position) {
    Runner* r = static_cast<Runner*>(runner);
    if (!r || !position) return TB_ERR_INVALID_ARG;
    *position = r->pos;
    return TB_OK;
}

extern "C" int tb_b200_runner_stream(void* runner, void** stream) {
    Runner* r = static_cast<Runner*>(runner);
    if (!r || !stream) return TB_ERR_INVALID_ARG;
    *stream = r->stream;
    return TB_OK;
}

extern "C" int tb_b200_runner_launches_per_token(void* runner, int* launches) {
    Runner* r = static_cast<Runner*>(runner);
    if (!r || !launches) return TB_ERR_INVALID_ARG;
    *launches = r->launches;
    return TB_OK;
}

extern "C" int tb_b200_runner_destroy(void* runner) {
    release(static_cast<Runner*>(runner));
    return TB_OK;
}
