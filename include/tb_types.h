/*
 * tb_types.h -- the tensorbit-run ABI types the b200 backend exchanges with
 * the engine: error codes, device and dtype enums, and the tensor descriptor.
 *
 * These are ABI-identical restatements of the engine's own declarations
 * (same names, values, field order and sizes), so that a TbTensor built by
 * the engine can be handed to this library unchanged:
 *   TbError   include/tensorbit/run/common.h:54-71
 *   TbDevice  include/tensorbit/run/common.h:77-83
 *   TbDtype   include/tensorbit/run/common.h:89-99
 *   TbTensor  include/tensorbit/run/tensor.h:47-54
 * When the engine's tensor.h is already included (its guard
 * TENSORBIT_RUN_TENSOR_H is defined) the engine's declarations are used and
 * only the additions below are made.
 *
 * Addition: TB_ERR_DEVICE (16), returned when a CUDA or NCCL call fails.
 */
#ifndef TB_TYPES_H
#define TB_TYPES_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifndef TENSORBIT_RUN_TENSOR_H

typedef enum {
    TB_OK = 0,
    TB_ERR_FILE_OPEN = 1,
    TB_ERR_FILE_READ = 2,
    TB_ERR_FILE_WRITE = 3,
    TB_ERR_FILE_SEEK = 4,
    TB_ERR_BAD_MAGIC = 5,
    TB_ERR_VERSION = 6,
    TB_ERR_OOM = 7,
    TB_ERR_INVALID_ARG = 8,
    TB_ERR_INVALID_SHAPE = 9,
    TB_ERR_UNSUPPORTED_DTYPE = 10,
    TB_ERR_TRUNCATED = 11,
    TB_ERR_LAYER_NOT_FOUND = 12,
    TB_ERR_JSON_PARSE = 13,
    TB_ERR_BACKEND_NOT_FOUND = 14,
    TB_ERR_MATH_ERROR = 15,
} TbError;

typedef enum {
    TB_DEVICE_CPU = 0,
    TB_DEVICE_CUDA = 1,
    TB_DEVICE_METAL = 2,
    TB_DEVICE_VULKAN = 3,
    TB_DEVICE_NPU = 4,
} TbDevice;

typedef enum {
    TB_DTYPE_F32 = 0,
    TB_DTYPE_F16 = 1,
    TB_DTYPE_BF16 = 2,
    TB_DTYPE_F64 = 3,
    TB_DTYPE_I32 = 4,
    TB_DTYPE_U8 = 5,
    TB_DTYPE_U32 = 6,
    TB_DTYPE_INT8 = 7,
    TB_DTYPE_INT4 = 8,
} TbDtype;

#define TB_MAX_RANK 8

typedef struct {
    void* data;
    size_t shape[TB_MAX_RANK];
    uint8_t rank;
    TbDtype dtype;
    TbDevice device;
    bool owns_data;
} TbTensor;

#endif /* !TENSORBIT_RUN_TENSOR_H */

/* A CUDA or NCCL call failed; tb_b200_last_error() has the message. */
#define TB_ERR_DEVICE 16

#ifdef __cplusplus
}
#endif
#endif /* TB_TYPES_H */
