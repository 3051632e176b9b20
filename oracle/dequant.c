/*
 * dequant.c -- CPU restatement of the reference's INT4/INT8 weight
 * dequantisation (tensorbit::run::Model::get_weight_fp32,
 * include/tensorbit/run/model.hpp:181-225).
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * n = rows * cols quantized weights, row-major; element i belongs to scale
 * group g = i / gs with gs = group_size, or n when group_size is 0
 * (model.hpp:197); its scale is scales[g] when g < the scale count, else 1
 * (model.hpp:205).  INT4 packs two weights per byte, element i in the low
 * nibble of byte i / 2 when i is even and the high nibble when odd, two's
 * complement (model.hpp:206-209); INT8 is one signed byte (model.hpp:213-
 * 215).  The weight is (float)q * scale: one f32 multiply.
 * tests/test_oracle.py pins this against the reference's own method
 * (oracle/pin_dequant.cpp).
 */
#include "oracle.h"

#define ORC_OK 0
#define ORC_ERR_INVALID_ARG 8
#define ORC_DT_INT8 7
#define ORC_DT_INT4 8

int orc_dequant_f32(int dtype, size_t n, const void* src, const float* scales, size_t n_scales,
                    uint32_t group_size, float* dst) {
    if ((dtype != ORC_DT_INT4 && dtype != ORC_DT_INT8) || (n && (src == NULL || dst == NULL)))
        return ORC_ERR_INVALID_ARG;
    const size_t gs = group_size > 0 ? group_size : n;
    for (size_t i = 0; i < n; ++i) {
        const size_t g = i / gs;
        const float scale = (g < n_scales) ? scales[g] : 1.0f;
        if (dtype == ORC_DT_INT4) {
            const uint8_t b = ((const uint8_t*)src)[i / 2];
            const int nib = (i & 1) ? (b >> 4) : (b & 0xF);
            dst[i] = (nib & 8) ? (float)(nib - 16) * scale : (float)nib * scale;
        } else {
            dst[i] = (float)((const int8_t*)src)[i] * scale;
        }
    }
    return ORC_OK;
}
