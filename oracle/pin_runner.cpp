// pin_runner.cpp -- the reference's own single-token decoder forward
// (tensorbit::run::TransformerRunner::forward,
// include/tensorbit/run/ops.hpp:79-288) over an in-memory model, for
// pinning the oracle's restatement (runner.c).
//
// TEST INFRASTRUCTURE ONLY.  Built by oracle/Makefile into oracle/_ref/
// against the reference tree's headers, src/model.c, src/ops/*.c and the CPU
// backend (src/backend/cpu/*.c), all unmodified.  The model is one blob of
// .tb records (a 4096-byte TBHeader, the f32 weights, then the mask bytes),
// one TbLayerDesc per record, named as the runner looks them up
// (ops.hpp:84-103, 259-271).  The runner always takes the sparse path for a
// projection (Model::get_mask never comes back empty), so a projection the
// caller gives without a mask gets all-ones 2:4 mask bytes here, which keeps
// every weight in the dense order.
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "tensorbit/run/ops.hpp"

extern "C" {
#include "oracle.h"
}

namespace {

struct Record {
    std::string name;
    size_t rows, cols;
    const float* w;
    std::vector<uint8_t> mask;
};

void add_proj(std::vector<Record>& recs, const std::string& name, const orc_lin& l) {
    if (!l.w) return;
    Record r{name, (size_t)l.rows, (size_t)l.cols, l.w, {}};
    const size_t nmask = (size_t)l.rows * ((size_t)l.cols / 4);
    if (l.mask)
        r.mask.assign(l.mask, l.mask + nmask);
    else
        r.mask.assign(nmask, 0x0F);
    recs.push_back(std::move(r));
}

void add_vec(std::vector<Record>& recs, const std::string& name, const float* w, size_t n) {
    if (w) recs.push_back(Record{name, n, 0, w, {}});
}

}  // namespace

extern "C" int pin_runner_run(const orc_runner_cfg* c, const orc_model* m, int n_tokens,
                              const int32_t* tokens, float* logits) {
    using namespace tensorbit::run;
    std::vector<Record> recs;
    const size_t H = (size_t)c->hidden, V = (size_t)c->vocab;
    add_vec(recs, "model.embed_tokens.weight", m->embed, V * H);
    recs.back().rows = V;
    recs.back().cols = H;
    for (int l = 0; l < c->layers; l++) {
        const orc_layer& ly = m->layers[l];
        const std::string p = "model.layers." + std::to_string(l) + ".";
        add_proj(recs, p + "self_attn.q_proj.weight", ly.q);
        add_proj(recs, p + "self_attn.k_proj.weight", ly.k);
        add_proj(recs, p + "self_attn.v_proj.weight", ly.v);
        add_proj(recs, p + "self_attn.o_proj.weight", ly.o);
        add_proj(recs, p + "mlp.gate_proj.weight", ly.gate);
        add_proj(recs, p + "mlp.up_proj.weight", ly.up);
        add_proj(recs, p + "mlp.down_proj.weight", ly.down);
        add_vec(recs, p + "input_layernorm.weight", ly.in_norm, H);
        add_vec(recs, p + "post_attention_layernorm.weight", ly.post_norm, H);
    }
    add_vec(recs, "model.norm.weight", m->final_norm, H);
    if (m->lm_head) {
        add_vec(recs, "lm_head.weight", m->lm_head, V * H);
        recs.back().rows = V;
        recs.back().cols = H;
    }

    // one blob: per record a header, the weights, the mask bytes
    std::vector<size_t> offs;
    size_t total = 0;
    for (const Record& r : recs) {
        offs.push_back(total);
        const size_t nw = r.cols ? r.rows * r.cols : r.rows;
        total += TB_HEADER_SIZE + nw * sizeof(float) + r.mask.size();
        total = (total + 63) & ~(size_t)63;
    }
    std::vector<uint8_t> blob(total, 0);
    Model model;
    TbModel* cm = model.c_model();
    cm->layers = static_cast<TbLayerDesc*>(std::calloc(recs.size(), sizeof(TbLayerDesc)));
    if (!cm->layers) return 7;
    cm->num_layers = (int)recs.size();
    for (size_t i = 0; i < recs.size(); i++) {
        const Record& r = recs[i];
        const size_t nw = r.cols ? r.rows * r.cols : r.rows;
        TBHeader hdr;
        std::memset(&hdr, 0, sizeof hdr);
        hdr.magic = TB_MAGIC;
        hdr.version = TB_VERSION;
        hdr.num_weights = nw;
        hdr.num_mask_bytes = r.mask.size();
        hdr.weights_offset = TB_HEADER_SIZE;
        hdr.masks_offset = TB_HEADER_SIZE + nw * sizeof(float);
        std::memcpy(blob.data() + offs[i], &hdr, sizeof hdr);
        std::memcpy(blob.data() + offs[i] + TB_HEADER_SIZE, r.w, nw * sizeof(float));
        if (!r.mask.empty())
            std::memcpy(blob.data() + offs[i] + hdr.masks_offset, r.mask.data(), r.mask.size());
        TbLayerDesc& d = cm->layers[i];
        std::snprintf(d.name, sizeof d.name, "%s", r.name.c_str());
        d.shape[0] = r.rows;
        d.shape[1] = r.cols;
        d.nm_n = r.mask.empty() ? 0 : 2;
        d.nm_m = r.mask.empty() ? 0 : 4;
        d.dtype = TB_DTYPE_F32;
        d.num_weights = nw;
        d.num_mask_bytes = r.mask.size();
        d.tbm_offset = offs[i];
    }
    cm->mapped_data = blob.data();
    cm->mapped_size = blob.size();
    cm->owns_mapping = false;
    TbModelConfig& mc = cm->config;
    std::snprintf(mc.architecture, sizeof mc.architecture, "llama");
    mc.hidden_size = c->hidden;
    mc.num_heads = c->n_heads;
    mc.num_kv_heads = c->n_kv_heads;
    mc.intermediate_size = c->intermediate;
    mc.vocab_size = c->vocab;
    mc.max_seq_len = c->max_seq;
    mc.num_layers = c->layers;
    mc.norm_eps = c->norm_eps;
    mc.rope_theta = c->rope_theta;
    mc.head_dim = c->head_dim;

    BackendRegistry::instance().init();
    int rc = 0;
    {
        TransformerRunner runner(model);
        runner.init_state();
        for (int t = 0; t < n_tokens; t++) {
            const float* lg = runner.forward(tokens[t]);
            if (!lg) {
                rc = 8;
                break;
            }
            std::memcpy(logits + (size_t)t * V, lg, V * sizeof(float));
        }
    }
    cm->mapped_data = nullptr;  // the blob is ours
    cm->mapped_size = 0;
    return rc;
}
