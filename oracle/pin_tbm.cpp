// pin_tbm.cpp -- the reference's own .tbm container code, for checking the
// device loader (tb_b200_tbm_*) against it.
//
// TEST INFRASTRUCTURE ONLY.  Built by oracle/Makefile into oracle/_ref/
// against the reference tree's headers, src/model.c, src/ops/*.c and the CPU
// backend, all unmodified.  Exposes:
//   pin_tbm_create  the reference's writer, tb_tbm_create (src/model.c:747-860);
//   pin_tbm_open / _count / _info / _close
//                   the reference's loader, tb_model_load_tbm
//                   (src/model.c:482-580), and its zero-copy views of each
//                   tensor (src/model.c:681-739), with their return codes;
//   pin_tbm_runner  the reference's TransformerRunner::forward
//                   (include/tensorbit/run/ops.hpp:79-288) over a model
//                   loaded from the file by Model::load_tbm.
#include <cstdint>
#include <cstring>

#include "tensorbit/run/ops.hpp"

extern "C" {

struct pin_tbm_layer {
    const char* name;
    uint64_t rows, cols;
    int nm_n, nm_m, dtype;
    const void* w;
    uint64_t w_bytes;
    const uint8_t* mask;
    uint64_t mask_bytes;
};

int pin_tbm_create(const char* path, const TbModelConfig* cfg, int n,
                   const pin_tbm_layer* ls) {
    TbLayerInput* in = static_cast<TbLayerInput*>(calloc((size_t)n, sizeof(TbLayerInput)));
    if (!in) return TB_ERR_OOM;
    for (int i = 0; i < n; ++i) {
        snprintf(in[i].name, sizeof in[i].name, "%s", ls[i].name);
        in[i].shape[0] = ls[i].rows;
        in[i].shape[1] = ls[i].cols;
        in[i].nm_n = ls[i].nm_n;
        in[i].nm_m = ls[i].nm_m;
        in[i].dtype = static_cast<TbDtype>(ls[i].dtype);
        in[i].weight_data = ls[i].w;
        in[i].weight_byte_size = ls[i].w_bytes;
        in[i].mask_data = ls[i].mask;
        in[i].mask_byte_size = ls[i].mask_bytes;
    }
    const int rc = tb_tbm_create(path, cfg, in, n);
    free(in);
    return rc;
}

struct pin_tbm_info {
    char name[128];
    uint64_t shape[2];
    int dtype;
    uint32_t nm_n, nm_m;
    uint64_t num_weights, num_mask_bytes, scale_count;
    uint32_t group_size;
    const void* w;
    const void* m;
    const void* s;
    int rc_w, rc_m, rc_s;
};

int pin_tbm_open(const char* path, void** h) {
    TbModel* m = static_cast<TbModel*>(calloc(1, sizeof(TbModel)));
    if (!m) return TB_ERR_OOM;
    const int rc = tb_model_load_tbm(m, path);
    if (rc != TB_OK) {
        free(m);
        return rc;
    }
    *h = m;
    return TB_OK;
}

int pin_tbm_config(void* h, TbModelConfig* out) {
    *out = static_cast<TbModel*>(h)->config;
    return TB_OK;
}

int pin_tbm_count(void* h) { return static_cast<TbModel*>(h)->num_layers; }

int pin_tbm_info(void* h, int i, pin_tbm_info* out) {
    const TbModel* m = static_cast<TbModel*>(h);
    if (i < 0 || i >= m->num_layers) return TB_ERR_LAYER_NOT_FOUND;
    const TbLayerDesc& d = m->layers[i];
    memset(out, 0, sizeof *out);
    snprintf(out->name, sizeof out->name, "%s", d.name);
    out->shape[0] = d.shape[0];
    out->shape[1] = d.shape[1];
    out->dtype = (int)d.dtype;
    out->nm_n = d.nm_n;
    out->nm_m = d.nm_m;
    out->num_weights = d.num_weights;
    out->num_mask_bytes = d.num_mask_bytes;
    out->scale_count = d.scale_count;
    out->group_size = d.group_size;
    TbTensor t;
    out->rc_w = tb_model_get_weight_tensor(m, i, &t);
    if (out->rc_w == TB_OK) out->w = t.data;
    out->rc_m = tb_model_get_mask_tensor(m, i, &t);
    if (out->rc_m == TB_OK) out->m = t.data;
    out->rc_s = tb_model_get_scale_tensor(m, i, &t);
    if (out->rc_s == TB_OK) out->s = t.data;
    return TB_OK;
}

void pin_tbm_close(void* h) {
    TbModel* m = static_cast<TbModel*>(h);
    tb_model_free(m);
    free(m);
}

int pin_tbm_runner(const char* path, int n_tokens, const int32_t* tokens, float* logits,
                   int vocab) {
    using namespace tensorbit::run;
    auto loaded = Model::load_tbm(path);
    if (!loaded) return TB_ERR_FILE_READ;
    Model& model = *loaded;
    BackendRegistry::instance().init();
    TransformerRunner runner(model);
    runner.init_state();
    for (int t = 0; t < n_tokens; t++) {
        const float* lg = runner.forward(tokens[t]);
        if (!lg) return TB_ERR_INVALID_ARG;
        memcpy(logits + (size_t)t * vocab, lg, (size_t)vocab * sizeof(float));
    }
    return TB_OK;
}

}  // extern "C"
