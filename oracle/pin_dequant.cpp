// pin_dequant.cpp -- the reference's own INT4/INT8 dequantisation
// (tensorbit::run::Model::get_weight_fp32, include/tensorbit/run/model.hpp:
// 181-225), called on an in-memory .tb blob, for pinning the oracle's
// restatement (dequant.c).
//
// TEST INFRASTRUCTURE ONLY.  Built by oracle/Makefile into oracle/_ref/
// against the reference tree's headers and src/model.c.  The blob holds the
// .tb header (magic, weights offset), the quantized weights and the scales
// right after them, which is where tb_model_get_scale_tensor looks
// (src/model.c:716-739); one TbLayerDesc describes it.
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "tensorbit/run/model.hpp"

extern "C" int pin_dequant_f32(int dtype, int64_t rows, int64_t cols, const void* qdata,
                               const float* scales, int64_t n_scales, uint32_t group_size,
                               float* out) {
    const size_t n = (size_t)rows * (size_t)cols;
    const size_t wbytes = dtype == TB_DTYPE_INT4 ? (n + 1) / 2 : n;
    std::vector<uint8_t> blob(TB_HEADER_SIZE + wbytes + (size_t)n_scales * sizeof(float));
    TBHeader hdr;
    std::memset(&hdr, 0, sizeof hdr);
    hdr.magic = TB_MAGIC;
    hdr.weights_offset = TB_HEADER_SIZE;
    std::memcpy(blob.data(), &hdr, sizeof hdr);
    std::memcpy(blob.data() + TB_HEADER_SIZE, qdata, wbytes);
    if (n_scales) std::memcpy(blob.data() + TB_HEADER_SIZE + wbytes, scales, n_scales * sizeof(float));

    tensorbit::run::Model m;
    TbModel* c = m.c_model();
    c->layers = static_cast<TbLayerDesc*>(std::calloc(1, sizeof(TbLayerDesc)));  // freed by ~Model
    if (!c->layers) return 7;
    c->num_layers = 1;
    TbLayerDesc& l = c->layers[0];
    l.shape[0] = (size_t)rows;
    l.shape[1] = (size_t)cols;
    l.dtype = (TbDtype)dtype;
    l.num_weights = n;
    l.scale_count = (size_t)n_scales;
    l.group_size = group_size;
    l.tbm_offset = 0;
    c->mapped_data = blob.data();
    c->mapped_size = blob.size();
    c->owns_mapping = false;
    tensorbit::run::Tensor t = m.get_weight_fp32(0);
    if (!t.f32()) return 8;
    std::memcpy(out, t.f32(), n * sizeof(float));
    return 0;
}
