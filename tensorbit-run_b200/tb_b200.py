"""Python binding of libtb_b200.so over its C ABI (include/tb_b200.h,
include/tb_backend.h), for tests, benchmarks and Python hosts.

Device buffers are torch CUDA tensors (torch provides allocation, streams
and torch.distributed; the arithmetic is the library's sm_100a kernels).
Every call goes through ctypes to the C entry point of the same name and
raises ``TbError`` on a nonzero TbError code.  There is no fallback path:
if the library is missing, ``lib()`` raises.

Dtype codes follow TbDtype (F32 = 0, BF16 = 2).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libtb_b200.so")

F32, F16, BF16, I32 = 0, 1, 2, 4
DEVICE_CPU, DEVICE_CUDA = 0, 1
FLAG_TOKEN_RANGE = 0x1
FLAG_WAIT_TIMEOUT = 0x2

# TbOpType values (include/tb_backend.h)
OP = dict(SPARSE_LINEAR=0, DENSE_LINEAR=1, RMS_NORM=2, LAYER_NORM=3, GELU=4, SILU=5, SOFTMAX=6,
          ATTENTION_QKV=7, SCALED_DOT_PRODUCT=8, ROPE=9, RESIDUAL_ADD=10, EMBEDDING=11, CONV2D=12,
          RESIDUAL_RMS_NORM=13, SWIGLU=14, ARGMAX=15, ROPE_ROWS=16, LAYER_CHAIN=17, COUNT=18)

ERRORS = {0: "ok", 7: "out of memory", 8: "invalid argument", 9: "invalid shape",
          10: "unsupported dtype", 14: "backend not found", 16: "device error"}


class TbError(RuntimeError):
    def __init__(self, code: int, what: str, detail: str = ""):
        self.code = code
        msg = f"{what}: TbError {code} ({ERRORS.get(code, 'error')})"
        super().__init__(msg + (f": {detail}" if detail else ""))


class TbTensor(C.Structure):
    """ABI image of TbTensor (include/tb_types.h)."""
    _fields_ = [("data", C.c_void_p), ("shape", C.c_size_t * 8), ("rank", C.c_uint8),
                ("dtype", C.c_int), ("device", C.c_int), ("owns_data", C.c_bool)]


class LayerChain(C.Structure):
    """ABI image of TbB200LayerChain (include/tb_b200.h)."""
    _fields_ = [("dtype", C.c_int), ("rows", C.c_int64),
                ("hidden", C.c_int64), ("x", C.c_void_p), ("residual", C.c_void_p),
                ("norm_weight", C.c_void_p), ("h_out", C.c_void_p), ("y", C.c_void_p),
                ("eps", C.c_float),
                ("n_q_heads", C.c_int), ("n_kv_heads", C.c_int), ("head_dim", C.c_int),
                ("q", C.c_void_p), ("k", C.c_void_p), ("positions", C.c_void_p),
                ("theta", C.c_float), ("rope_table", C.c_void_p),
                ("rope_table_positions", C.c_int),
                ("intermediate", C.c_int64), ("gate", C.c_void_p), ("up", C.c_void_p),
                ("act_out", C.c_void_p)]


class RopeRowsParams(C.Structure):
    _fields_ = [("positions", C.c_void_p), ("theta", C.c_float), ("head_dim", C.c_int),
                ("max_position", C.c_int)]


class LayerChainParams(C.Structure):
    _fields_ = [("eps", C.c_float), ("positions", C.c_void_p), ("theta", C.c_float),
                ("head_dim", C.c_int), ("max_position", C.c_int)]


_lib = None
vp, i64, i32, f32 = C.c_void_p, C.c_int64, C.c_int, C.c_float
P = C.POINTER

INT8, INT4 = 7, 8  # TbDtype codes of quantized weights
ATTN_REFERENCE, ATTN_STANDARD = 0, 1
FLAG_POSITION_RANGE = 0x4
PROJECTIONS = ("q", "k", "v", "o", "gate", "up", "down")


class Weight(C.Structure):  # TbB200Weight
    _fields_ = [("data", vp), ("dtype", i32), ("rows", i64), ("cols", i64), ("mask", vp),
                ("scales", vp), ("n_scales", i64), ("group_size", C.c_uint32)]


class RunnerLayer(C.Structure):  # TbB200RunnerLayer
    _fields_ = [(n, Weight) for n in PROJECTIONS] + [("input_norm", vp), ("post_norm", vp)]


class RunnerDesc(C.Structure):  # TbB200RunnerDesc
    _fields_ = [(n, i32) for n in ("hidden", "n_heads", "n_kv_heads", "head_dim", "intermediate",
                                   "vocab", "max_seq", "layers")] + [
        ("norm_eps", f32), ("rope_theta", f32), ("attention", i32), ("use_graph", i32),
        ("embed", Weight), ("final_norm", vp), ("lm_head", Weight), ("layer", P(RunnerLayer))]

class TbmConfig(C.Structure):  # TbB200TbmConfig
    _fields_ = [("architecture", C.c_char * 64)] + [
        (n, i32) for n in ("hidden_size", "num_heads", "num_kv_heads", "intermediate_size",
                           "vocab_size", "max_seq_len", "num_layers")] + [
        ("norm_eps", f32), ("rope_theta", f32), ("head_dim", i32)]


class TbmTensor(C.Structure):  # TbB200TbmTensor
    _fields_ = [("name", C.c_char * 128), ("shape", i64 * 2), ("dtype", i32),
                ("nm_n", C.c_uint32), ("nm_m", C.c_uint32), ("num_weights", i64),
                ("num_mask_bytes", i64), ("scale_count", i64), ("group_size", C.c_uint32),
                ("weights", vp), ("mask", vp), ("scales", vp), ("weight_bytes", i64)]


# name -> (restype, argtypes); every entry point of include/tb_b200.h and tb_backend.h.
SIGNATURES = {
    "tb_b200_version": (i32, []),
    "tb_b200_last_error": (C.c_char_p, []),
    "tb_b200_launch_count": (C.c_ulonglong, []),
    "tb_b200_device_count": (i32, [P(i32)]),
    "tb_b200_set_device": (i32, [i32]),
    "tb_b200_get_device": (i32, [P(i32)]),
    "tb_b200_malloc": (i32, [P(vp), C.c_size_t]),
    "tb_b200_free": (i32, [vp]),
    "tb_b200_malloc_host": (i32, [P(vp), C.c_size_t]),
    "tb_b200_free_host": (i32, [vp]),
    "tb_b200_memcpy_h2d": (i32, [vp, vp, C.c_size_t, vp]),
    "tb_b200_memcpy_d2h": (i32, [vp, vp, C.c_size_t, vp]),
    "tb_b200_memcpy_d2d": (i32, [vp, vp, C.c_size_t, vp]),
    "tb_b200_memset": (i32, [vp, i32, C.c_size_t, vp]),
    "tb_b200_set_stream": (i32, [vp]),
    "tb_b200_get_stream": (vp, []),
    "tb_b200_stream_sync": (i32, [vp]),
    "tb_b200_sync": (i32, []),
    "tb_b200_stage_h2d": (i32, [vp, C.c_size_t, P(vp), vp]),
    "tb_b200_stage_release": (i32, [vp, vp]),
    "tb_b200_is_device_ptr": (i32, [vp, P(i32)]),
    "tb_b200_check_status": (i32, [vp, P(C.c_uint)]),
    "tb_b200_residual_rms_norm": (i32, [i32, i64, i64, vp, vp, vp, vp, vp, f32, vp]),
    "tb_b200_rms_norm": (i32, [i32, i64, i64, vp, vp, vp, f32, vp]),
    "tb_b200_residual_add": (i32, [i32, i64, vp, vp, vp, vp]),
    "tb_b200_silu": (i32, [i32, i64, vp, vp, vp]),
    "tb_b200_gelu": (i32, [i32, i64, vp, vp, vp]),
    "tb_b200_swiglu": (i32, [i32, i64, vp, vp, vp, vp]),
    "tb_b200_rope_table": (i32, [f32, i32, i32, vp, vp]),
    "tb_b200_rope_rows": (i32, [i32, i64, i32, i32, i32, vp, vp, vp, f32, vp, i32, vp]),
    "tb_b200_rope": (i32, [i32, i32, i32, i32, vp, vp, i32, f32, vp]),
    "tb_b200_softmax": (i32, [i32, i64, i64, vp, vp, vp, vp]),
    "tb_b200_sample_temperature": (i32, [i64, i64, vp, f32, vp, vp, vp]),
    "tb_b200_dequant": (i32, [i32, i64, vp, vp, i64, C.c_uint32, i32, vp, vp]),
    "tb_b200_sparse_linear": (i32, [i64, i64, vp, vp, vp, vp, vp, i32, i32, vp]),
    "tb_b200_dense_linear": (i32, [i64, i64, vp, vp, vp, vp, vp]),
    "tb_b200_argmax": (i32, [i32, i64, i64, vp, vp, vp]),
    "tb_b200_embedding": (i32, [i32, i64, i64, i64, vp, vp, vp, vp]),
    "tb_b200_embedding_host_ids": (i32, [i32, i64, i64, i64, vp, vp, vp, vp]),
    "tb_b200_embedding_host_ids_static": (i32, [i32, i64, i64, i64, vp, vp, vp, vp]),
    "tb_b200_layer_chain": (i32, [P(LayerChain), vp]),
    "tb_b200_sparse24_pack": (i32, [i64, i64, vp, vp, vp, vp, vp, vp]),
    "tb_b200_sparse24_linear": (i32, [i64, i64, vp, vp, vp, vp, vp, vp]),
    "tb_b200_decode_attention": (i32, [i32, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp]),
    "tb_b200_runner_create": (i32, [P(RunnerDesc), P(vp)]),
    "tb_b200_runner_forward": (i32, [vp, C.c_int32, P(vp)]),
    "tb_b200_runner_logits": (i32, [vp, vp]),
    "tb_b200_runner_reset": (i32, [vp]),
    "tb_b200_runner_position": (i32, [vp, P(i32)]),
    "tb_b200_runner_stream": (i32, [vp, P(vp)]),
    "tb_b200_runner_launches_per_token": (i32, [vp, P(i32)]),
    "tb_b200_runner_destroy": (i32, [vp]),
    "tb_b200_tbm_load": (i32, [C.c_char_p, vp, P(vp)]),
    "tb_b200_tbm_config": (i32, [vp, P(TbmConfig)]),
    "tb_b200_tbm_count": (i32, [vp, P(i32)]),
    "tb_b200_tbm_find": (i32, [vp, C.c_char_p, P(i32)]),
    "tb_b200_tbm_tensor": (i32, [vp, i32, P(TbmTensor)]),
    "tb_b200_tbm_runner_desc": (i32, [vp, i32, i32, P(RunnerDesc), P(RunnerLayer), i32]),
    "tb_b200_tbm_free": (i32, [vp]),
    "tb_b200_partition": (i32, [i64, i32, i32, P(i64), P(i64)]),
    "tb_b200_shard_plan": (i32, [i64, i64, i32, i32, vp, vp, vp, vp, vp, vp, vp, P(i64)]),
    "tb_b200_comm_unique_id": (i32, [vp]),
    "tb_b200_comm_init": (i32, [i32, i32, vp, i32]),
    "tb_b200_comm_destroy": (i32, []),
    "tb_b200_comm_info": (i32, [P(i32), P(i32)]),
    "tb_b200_comm_wait": (i32, [vp]),
    "tb_b200_selftest_wait": (i32, [i32, C.c_uint32, vp]),
    "tb_b200_comm_window_alloc": (i32, [C.c_size_t, P(vp)]),
    "tb_b200_comm_window_free": (i32, [vp]),
    "tb_b200_embedding_sharded_window": (i32, [i32, i64, i64, i64, vp, vp, vp, vp]),
    "tb_b200_embedding_sharded": (i32, [i32, i64, i64, i64, vp, vp, vp, vp]),
    "tb_b200_embedding_sharded_p2p": (i32, [i32, i64, i64, i64, vp, P(vp), i32, vp, vp]),
    "tb_b200_p2p_export": (i32, [vp, vp, P(i64)]),
    "tb_b200_p2p_import": (i32, [vp, i64, P(vp)]),
    "tb_b200_p2p_close": (i32, [vp, i64]),
    # registry (include/tb_backend.h)
    "tb_backend_register": (i32, [vp]),
    "tb_backend_register_device": (i32, [vp, i32]),
    "tb_backend_get_best": (vp, [i32]),
    "tb_backend_get_best_device": (vp, [i32, i32]),
    "tb_backend_count": (i32, []),
    "tb_backend_get": (vp, [i32]),
    "tb_backend_reset": (None, []),
    "tb_backend_b200_init": (i32, []),
    "tb_dispatch_sparse_linear": (i32, [vp, vp, vp, vp, vp]),
    "tb_dispatch_dense_linear": (i32, [vp, vp, vp, vp]),
    "tb_dispatch_rms_norm": (i32, [vp, vp, vp, f32]),
    "tb_dispatch_layer_norm": (i32, [vp, vp, vp, vp, f32]),
    "tb_dispatch_gelu": (i32, [vp, vp]),
    "tb_dispatch_silu": (i32, [vp, vp]),
    "tb_dispatch_softmax": (i32, [vp, vp, vp]),
    "tb_dispatch_attention_qkv": (i32, [vp] * 10 + [i32, i32, i32]),
    "tb_dispatch_scaled_dot_product": (i32, [vp, vp, vp, vp, vp, f32, C.c_bool]),
    "tb_dispatch_rope": (i32, [vp, vp, i32, f32, i32]),
    "tb_dispatch_residual_add": (i32, [vp, vp, vp]),
    "tb_dispatch_embedding": (i32, [vp, vp, i32, vp]),
    "tb_dispatch_conv2d": (i32, [vp, vp, vp, vp, i32, i32]),
    "tb_dispatch_residual_rms_norm": (i32, [vp, vp, vp, vp, vp, f32]),
    "tb_dispatch_swiglu": (i32, [vp, vp, vp]),
    "tb_dispatch_argmax": (i32, [vp, vp]),
    "tb_dispatch_rope_rows": (i32, [vp, vp, vp, f32, i32, i32]),
    "tb_dispatch_layer_chain": (i32, [vp] * 10 + [P(LayerChainParams)]),
}


def build() -> None:
    """Compile lib/libtb_b200.so (nvcc, sm_100a)."""
    out = subprocess.run(["make", "-C", HERE, "-j8"], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("libtb_b200 build failed:\n" + out.stdout[-4000:] + out.stderr[-4000:])


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is not built (run __graft_entry__.build())")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    s = lib().tb_b200_last_error()
    return s.decode() if s else ""


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise TbError(rc, what, last_error())


# ------------------------------------------------------------- torch glue
def _torch():
    import torch
    return torch


def dtype_code(t) -> int:
    torch = _torch()
    if t.dtype == torch.float32:
        return F32
    if t.dtype == torch.bfloat16:
        return BF16
    if t.dtype == torch.int32:
        return I32
    raise TypeError(f"unsupported dtype {t.dtype}")


def ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def cur_stream():
    torch = _torch()
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _dev(*ts):
    for t in ts:
        if t is not None and not (t.is_cuda and t.is_contiguous()):
            raise ValueError("expected contiguous CUDA tensors")


def residual_rms_norm(x, residual, weight, eps, h_out=None, y=None, stream=None):
    torch = _torch()
    y = torch.empty_like(x) if y is None else y
    _dev(x, residual, weight, h_out, y)
    rows, cols = (x.numel() // x.shape[-1], x.shape[-1]) if x.dim() else (1, 1)
    check(lib().tb_b200_residual_rms_norm(dtype_code(x), rows, cols, ptr(x), ptr(residual),
                                          ptr(weight), ptr(h_out), ptr(y), eps,
                                          stream or cur_stream()), "residual_rms_norm")
    return h_out, y


def rms_norm(x, weight, eps, y=None, stream=None):
    torch = _torch()
    y = torch.empty_like(x) if y is None else y
    _dev(x, weight, y)
    rows, cols = x.numel() // x.shape[-1], x.shape[-1]
    check(lib().tb_b200_rms_norm(dtype_code(x), rows, cols, ptr(x), ptr(weight), ptr(y), eps,
                                 stream or cur_stream()), "rms_norm")
    return y


def residual_add(x, residual, y=None, stream=None):
    torch = _torch()
    y = torch.empty_like(x) if y is None else y
    _dev(x, residual, y)
    check(lib().tb_b200_residual_add(dtype_code(x), x.numel(), ptr(x), ptr(residual), ptr(y),
                                     stream or cur_stream()), "residual_add")
    return y


def silu(x, y=None, stream=None):
    torch = _torch()
    y = torch.empty_like(x) if y is None else y
    _dev(x, y)
    check(lib().tb_b200_silu(dtype_code(x), x.numel(), ptr(x), ptr(y), stream or cur_stream()),
          "silu")
    return y


def gelu(x, y=None, stream=None):
    torch = _torch()
    y = torch.empty_like(x) if y is None else y
    _dev(x, y)
    check(lib().tb_b200_gelu(dtype_code(x), x.numel(), ptr(x), ptr(y), stream or cur_stream()),
          "gelu")
    return y


def swiglu(gate, up, out=None, stream=None):
    torch = _torch()
    out = torch.empty_like(gate) if out is None else out
    _dev(gate, up, out)
    check(lib().tb_b200_swiglu(dtype_code(gate), gate.numel(), ptr(gate), ptr(up), ptr(out),
                               stream or cur_stream()), "swiglu")
    return out


def rope_table(theta, head_dim, n_positions, device=None):
    torch = _torch()
    t = torch.empty((n_positions, head_dim), dtype=torch.float32,
                    device=device or torch.cuda.current_device())
    check(lib().tb_b200_rope_table(theta, head_dim, n_positions, ptr(t), cur_stream()),
          "rope_table")
    return t


def rope_rows(q, k, positions, theta, table=None, stream=None):
    """In place on q [R, Hq, d] and k [R, Hkv, d]; positions int32 [R] on the device."""
    _dev(q, k, positions, table)
    rows, hq, d = q.shape
    hkv = k.shape[1]
    check(lib().tb_b200_rope_rows(dtype_code(q), rows, hq, hkv, d, ptr(q), ptr(k), ptr(positions),
                                  theta, ptr(table), 0 if table is None else table.shape[0],
                                  stream or cur_stream()), "rope_rows")
    return q, k


def rope(q, k, position, theta, stream=None):
    """Single token: q [Hq, d], k [Hkv, d], in place."""
    _dev(q, k)
    check(lib().tb_b200_rope(dtype_code(q), q.shape[0], k.shape[0], q.shape[-1], ptr(q), ptr(k),
                             position, theta, stream or cur_stream()), "rope")
    return q, k


def softmax(x, mask=None, y=None, stream=None):
    torch = _torch()
    y = torch.empty_like(x) if y is None else y
    _dev(x, mask, y)
    rows, cols = x.numel() // x.shape[-1], x.shape[-1]
    check(lib().tb_b200_softmax(dtype_code(x), rows, cols, ptr(x), ptr(mask), ptr(y),
                                stream or cur_stream()), "softmax")
    return y


def argmax(x, out=None, stream=None):
    torch = _torch()
    rows, cols = x.numel() // x.shape[-1], x.shape[-1]
    out = torch.empty(rows, dtype=torch.int32, device=x.device) if out is None else out
    _dev(x, out)
    check(lib().tb_b200_argmax(dtype_code(x), rows, cols, ptr(x), ptr(out),
                               stream or cur_stream()), "argmax")
    return out


def sample_temperature(logits, temperature, uniforms, out=None, stream=None):
    """Index drawn per row of f32 logits at the given uniform (float64 device
    tensor, one per row), as the reference's sample_temperature draws it."""
    torch = _torch()
    rows, cols = logits.numel() // logits.shape[-1], logits.shape[-1]
    out = torch.empty(rows, dtype=torch.int32, device=logits.device) if out is None else out
    _dev(logits, out)
    u = None if uniforms is None else ptr(uniforms)
    check(lib().tb_b200_sample_temperature(rows, cols, ptr(logits), temperature, u, ptr(out),
                                           stream or cur_stream()), "sample_temperature")
    return out


def dequant(src_dtype, n, q, scales, group_size, out_dtype=F32, out=None, stream=None):
    """n INT4 (src_dtype 8) / INT8 (7) weights in the uint8 device tensor q
    to f32 or bf16 with per-group f32 scales (Model::get_weight_fp32)."""
    torch = _torch()
    if out is None:
        dt = torch.float32 if out_dtype == F32 else torch.bfloat16
        out = torch.empty(n, dtype=dt, device=q.device)
    _dev(q, out)
    check(lib().tb_b200_dequant(src_dtype, n, ptr(q), ptr(scales) if scales is not None else None,
                                0 if scales is None else scales.numel(), group_size, out_dtype,
                                ptr(out), stream or cur_stream()), "dequant")
    return out


def linear(x, w, mask=None, bias=None, nm_n=2, nm_m=4, y=None, stream=None):
    """y = W x (+ bias) for an f32 vector x: N:M-masked when `mask` (uint8,
    one byte per M-group of a row) is given, else dense."""
    torch = _torch()
    out_f, in_f = w.shape
    y = torch.empty(out_f, dtype=torch.float32, device=w.device) if y is None else y
    _dev(x, w, y)
    b = ptr(bias) if bias is not None else None
    if mask is not None:
        rc = lib().tb_b200_sparse_linear(out_f, in_f, ptr(x), ptr(w), ptr(mask), b, ptr(y), nm_n,
                                         nm_m, stream or cur_stream())
    else:
        rc = lib().tb_b200_dense_linear(out_f, in_f, ptr(x), ptr(w), b, ptr(y),
                                        stream or cur_stream())
    check(rc, "linear")
    return y


def sparse24_pack(w, mask, stream=None):
    """Pack a 2:4-masked f32 [out, in] weight: (vals float32 [out, P, 4],
    idx uint8 [out, S], packable) with P = ceil((in / 4) / 2) and S = P
    rounded up to a multiple of 128."""
    torch = _torch()
    out_f, in_f = w.shape
    pairs = (in_f // 4 + 1) // 2
    vals = torch.empty((out_f, pairs, 4), dtype=torch.float32, device=w.device)
    idx = torch.empty((out_f, (pairs + 127) // 128 * 128), dtype=torch.uint8, device=w.device)
    flag = torch.zeros(1, dtype=torch.int32, device=w.device)
    _dev(w, mask)
    check(lib().tb_b200_sparse24_pack(out_f, in_f, ptr(w), ptr(mask), ptr(vals), ptr(idx),
                                      ptr(flag), stream or cur_stream()), "sparse24_pack")
    return vals, idx, int(flag.item()) == 0


def sparse24_linear(x, vals, idx, in_features, bias=None, y=None, stream=None):
    torch = _torch()
    out_f = vals.shape[0]
    y = torch.empty(out_f, dtype=torch.float32, device=x.device) if y is None else y
    _dev(x, vals, idx, y)
    check(lib().tb_b200_sparse24_linear(out_f, in_features, ptr(x), ptr(vals), ptr(idx),
                                        ptr(bias) if bias is not None else None, ptr(y),
                                        stream or cur_stream()), "sparse24_linear")
    return y


def embedding(ids, table, y=None, stream=None):
    torch = _torch()
    n = ids.numel()
    y = torch.empty((n, table.shape[1]), dtype=table.dtype, device=table.device) if y is None else y
    _dev(ids, table, y)
    check(lib().tb_b200_embedding(dtype_code(table), n, table.shape[1], table.shape[0], ptr(ids),
                                  ptr(table), ptr(y), stream or cur_stream()), "embedding")
    return y


def check_status(stream=None):
    flags = C.c_uint(0)
    rc = lib().tb_b200_check_status(stream or cur_stream(), C.byref(flags))
    return rc, flags.value


def layer_chain(chain: LayerChain, stream=None):
    check(lib().tb_b200_layer_chain(C.byref(chain), stream or cur_stream()), "layer_chain")


def make_chain(x=None, residual=None, norm_weight=None, h_out=None, y=None, eps=1e-5, q=None,
               k=None, positions=None, theta=10000.0, table=None, gate=None, up=None,
               act_out=None) -> LayerChain:
    c = LayerChain()
    ref = next(t for t in (x, q, gate) if t is not None)
    c.dtype = dtype_code(ref)
    c.rows = ref.shape[0]
    if x is not None:
        c.hidden, c.x, c.residual = x.shape[-1], ptr(x), ptr(residual)
        c.norm_weight, c.h_out, c.y, c.eps = ptr(norm_weight), ptr(h_out), ptr(y), eps
    if q is not None:
        c.n_q_heads, c.n_kv_heads, c.head_dim = q.shape[1], k.shape[1], q.shape[2]
        c.q, c.k, c.positions, c.theta = ptr(q), ptr(k), ptr(positions), theta
        c.rope_table = ptr(table)
        c.rope_table_positions = 0 if table is None else table.shape[0]
    if gate is not None:
        c.intermediate, c.gate, c.up, c.act_out = gate.shape[-1], ptr(gate), ptr(up), ptr(act_out)
    return c


def tensor(t, device=None) -> TbTensor:
    """TbTensor view of a torch tensor (no copy, owns_data = false)."""
    d = TbTensor()
    d.data = t.data_ptr()
    for i, s in enumerate(t.shape):
        d.shape[i] = s
    d.rank = t.dim()
    d.dtype = dtype_code(t)
    d.device = (DEVICE_CUDA if t.is_cuda else DEVICE_CPU) if device is None else device
    d.owns_data = False
    return d


# ------------------------------------------------------------ multi-GPU
def partition(total: int, parts: int, part: int):
    """[lo, hi) of part `part` when `total` items are split into `parts`."""
    lo, hi = C.c_int64(), C.c_int64()
    check(lib().tb_b200_partition(total, parts, part, C.byref(lo), C.byref(hi)), "partition")
    return lo.value, hi.value


def shard_plan(ids, vocab: int, nranks: int, rank: int):
    """The exchange plan of tb_b200_embedding_sharded for `rank` (host only):
    (send_counts, recv_counts, send_rows, recv_rows, local_dst, local_src) as
    numpy arrays, trimmed to their counts."""
    import numpy as np
    ids = np.ascontiguousarray(ids, np.int32)
    n = len(ids)
    sc = np.zeros(nranks, np.int64)
    rc = np.zeros(nranks, np.int64)
    bufs = [np.zeros(n + 1, np.int32) for _ in range(4)]
    nl = C.c_int64()
    check(lib().tb_b200_shard_plan(n, vocab, nranks, rank, ids.ctypes.data, sc.ctypes.data,
                                   rc.ctypes.data, *[b.ctypes.data for b in bufs], C.byref(nl)),
          "shard_plan")
    s, r, ld, ls = bufs
    return sc, rc, s[:sc.sum()], r[:rc.sum()], ld[:nl.value], ls[:nl.value]


def comm_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    check(lib().tb_b200_comm_unique_id(buf), "comm_unique_id")
    return buf.raw


def comm_init(nranks: int, rank: int, unique_id: bytes, device: int) -> None:
    buf = C.create_string_buffer(bytes(unique_id), 128)
    check(lib().tb_b200_comm_init(nranks, rank, buf, device), "comm_init")


def comm_destroy() -> None:
    check(lib().tb_b200_comm_destroy(), "comm_destroy")


def comm_wait(stream=None) -> int:
    """Bounded wait for the stream's queued work, exchanges included
    (tb_b200_comm_wait): TB_OK, or TB_ERR_DEVICE after aborting the
    communicator on an error or a timeout.  Returns the code."""
    return lib().tb_b200_comm_wait(stream or cur_stream())


def comm_window_alloc(nbytes: int) -> int:
    """Device address of `nbytes` of the communicator's symmetric memory
    (collective: every rank, same size, same order)."""
    p = vp()
    check(lib().tb_b200_comm_window_alloc(nbytes, C.byref(p)), "comm_window_alloc")
    return p.value


def comm_window_free(addr: int) -> None:
    check(lib().tb_b200_comm_window_free(vp(addr)), "comm_window_free")


def embedding_sharded_window(ids, shard_addr: int, vocab: int, dim: int, dtype, y=None,
                             stream=None):
    """Rows of `ids` (int32 CUDA tensor) from the vocab shards held in the
    communicator's symmetric memory (tb_b200_embedding_sharded_window)."""
    torch = _torch()
    _dev(ids)
    if y is None:
        y = torch.empty((ids.numel(), dim), dtype=dtype, device=ids.device)
    check(lib().tb_b200_embedding_sharded_window(dtype_code(y), ids.numel(), dim, vocab, ptr(ids),
                                                 vp(shard_addr), ptr(y), stream or cur_stream()),
          "embedding_sharded_window")
    return y


def comm_info():
    """(rank, nranks) of this process's communicator; (0, 0) without one."""
    rank, nranks = C.c_int(), C.c_int()
    check(lib().tb_b200_comm_info(C.byref(rank), C.byref(nranks)), "comm_info")
    return rank.value, nranks.value


def embedding_sharded(ids_host, table_shard, vocab: int, y_local=None, stream=None):
    """This rank's token part of the full-table gather, from its vocab shard
    (tb_b200_embedding_sharded).  ids_host: int32 numpy array of all tokens."""
    import numpy as np
    torch = _torch()
    rank, nranks = C.c_int(), C.c_int()
    check(lib().tb_b200_comm_info(C.byref(rank), C.byref(nranks)), "comm_info")
    ids = np.ascontiguousarray(ids_host, np.int32)
    lo, hi = partition(len(ids), nranks.value, rank.value)
    if y_local is None:
        y_local = torch.empty((hi - lo, table_shard.shape[1]), dtype=table_shard.dtype,
                              device=table_shard.device)
    check(lib().tb_b200_embedding_sharded(dtype_code(table_shard), len(ids), table_shard.shape[1],
                                          vocab, ids.ctypes.data, ptr(table_shard), ptr(y_local),
                                          stream or cur_stream()), "embedding_sharded")
    return y_local


P2P_HANDLE_BYTES = 64


def p2p_export(t):
    """(handle bytes, offset) of CUDA tensor t's allocation, for the other
    processes of the box to import (tb_b200_p2p_export)."""
    _dev(t)
    h = C.create_string_buffer(P2P_HANDLE_BYTES)
    off = C.c_int64()
    check(lib().tb_b200_p2p_export(ptr(t), h, C.byref(off)), "p2p_export")
    return h.raw, off.value


def p2p_import(handle: bytes, offset: int) -> int:
    """Device address, in this process, of a buffer another process exported."""
    p = vp()
    check(lib().tb_b200_p2p_import(C.create_string_buffer(bytes(handle), P2P_HANDLE_BYTES),
                                   offset, C.byref(p)), "p2p_import")
    return p.value


def p2p_close(addr: int, offset: int) -> None:
    check(lib().tb_b200_p2p_close(vp(addr), offset), "p2p_close")


def embedding_sharded_p2p(ids, shard_addrs, vocab: int, dim: int, dtype, y=None, stream=None):
    """The rows of `ids` (int32 CUDA tensor) gathered in one kernel from the
    vocab shards at `shard_addrs` (device addresses, rank order)
    (tb_b200_embedding_sharded_p2p)."""
    torch = _torch()
    _dev(ids)
    if ids.dtype != torch.int32:
        raise TypeError("ids must be int32")
    if y is None:
        y = torch.empty((ids.numel(), dim), dtype=dtype, device=ids.device)
    _dev(y)
    arr = (vp * len(shard_addrs))(*shard_addrs)
    check(lib().tb_b200_embedding_sharded_p2p(dtype_code(y), ids.numel(), dim, vocab, ptr(ids),
                                              arr, len(shard_addrs), ptr(y),
                                              stream or cur_stream()), "embedding_sharded_p2p")
    return y


# ------------------------------------------------ decoder forward (runner)
def decode_attention(q, k, v, k_cache, v_cache, position, n_heads, n_kv_heads,
                     mode=ATTN_REFERENCE, out=None, stream=None):
    """Single-token attention over one layer's f32 KV cache
    [max_seq, n_kv_heads * head_dim]; `position` a 1-element int32 device
    tensor.  Also writes k and v into cache row `position`."""
    torch = _torch()
    head_dim = q.numel() // n_heads
    out = torch.empty(n_heads * head_dim, dtype=torch.float32, device=q.device) if out is None else out
    _dev(q, k, v, k_cache, v_cache, position, out)
    check(lib().tb_b200_decode_attention(mode, n_heads, n_kv_heads, head_dim, k_cache.shape[0],
                                         ptr(position), ptr(q), ptr(k), ptr(v), ptr(k_cache),
                                         ptr(v_cache), ptr(out), stream or cur_stream()),
          "decode_attention")
    return out


class QuantWeight:
    """An INT4 (dtype INT4, two weights per byte, low nibble first) or INT8
    weight tensor [rows, cols] with per-group f32 scales, as a .tbm layer
    stores it."""

    def __init__(self, data, dtype, rows, cols, scales, group_size):
        self.data, self.dtype, self.rows, self.cols = data, dtype, rows, cols
        self.scales, self.group_size = scales, group_size


class Runner:
    """TransformerRunner (include/tensorbit/run/ops.hpp:33-288) on the device.

    cfg: dict with hidden, n_heads, n_kv_heads, head_dim, intermediate,
    vocab, max_seq, layers, norm_eps, rope_theta.  model: {"embed": W,
    "final_norm": v, "lm_head": W or None, "layers": [{"q": (W, mask), ...,
    "in_norm": v, "post_norm": v}]}, where W is an f32 numpy array (copied
    to the device), an f32 CUDA tensor (borrowed) or a QuantWeight, and a
    mask is uint8 2:4 group bytes or None (dense)."""

    def __init__(self, cfg, model, attention=ATTN_REFERENCE, use_graph=True):
        import numpy as np
        self._keep = []
        self.vocab = int(cfg["vocab"])

        def addr(a, dt=None):
            if a is None:
                return None
            if hasattr(a, "data_ptr"):
                self._keep.append(a)
                return a.data_ptr()
            a = np.ascontiguousarray(a, dtype=dt)
            self._keep.append(a)
            return a.ctypes.data

        def weight(w, mask=None):
            if w is None:
                return Weight()
            if isinstance(w, QuantWeight):
                sc = w.scales
                n_sc = 0 if sc is None else int(sc.numel() if hasattr(sc, "numel") else np.size(sc))
                return Weight(addr(w.data, np.uint8), w.dtype, w.rows, w.cols, addr(mask, np.uint8),
                              addr(sc, np.float32), n_sc, w.group_size)
            return Weight(addr(w, np.float32), F32, w.shape[0], w.shape[1], addr(mask, np.uint8),
                          None, 0, 0)

        n_layers = int(cfg["layers"])
        layers = (RunnerLayer * max(1, n_layers))()
        for i, ly in enumerate(model["layers"][:n_layers]):
            for n in PROJECTIONS:
                wm = ly.get(n)
                if wm is not None:
                    setattr(layers[i], n, weight(wm[0], wm[1] if len(wm) > 1 else None))
            layers[i].input_norm = addr(ly.get("in_norm"), np.float32)
            layers[i].post_norm = addr(ly.get("post_norm"), np.float32)
        d = RunnerDesc(*[int(cfg[n]) for n in ("hidden", "n_heads", "n_kv_heads", "head_dim",
                                               "intermediate", "vocab", "max_seq", "layers")],
                       float(cfg.get("norm_eps", 1e-5)), float(cfg.get("rope_theta", 10000.0)),
                       attention, 1 if use_graph else 0, weight(model["embed"]),
                       addr(model.get("final_norm"), np.float32), weight(model.get("lm_head")),
                       layers)
        h = vp()
        check(lib().tb_b200_runner_create(C.byref(d), C.byref(h)), "runner_create")
        self._h = h
        # host arrays were copied during create; device tensors stay borrowed
        self._keep = [a for a in self._keep if hasattr(a, "data_ptr")]

    @classmethod
    def from_desc(cls, desc, vocab, keep=()):
        """A runner from a filled RunnerDesc (e.g. tb_b200_tbm_runner_desc);
        `keep` holds whatever the descriptor points into."""
        self = cls.__new__(cls)
        self._keep = list(keep)
        self.vocab = int(vocab)
        h = vp()
        check(lib().tb_b200_runner_create(C.byref(desc), C.byref(h)), "runner_create")
        self._h = h
        return self

    def forward(self, token):
        """Run one token; returns the device logits address (valid until the
        next forward)."""
        out = vp()
        check(lib().tb_b200_runner_forward(self._h, int(token), C.byref(out)), "runner_forward")
        return out.value

    def logits(self):
        import numpy as np
        out = np.empty(self.vocab, dtype=np.float32)
        check(lib().tb_b200_runner_logits(self._h, out.ctypes.data), "runner_logits")
        return out

    def reset(self):
        check(lib().tb_b200_runner_reset(self._h), "runner_reset")

    @property
    def position(self):
        p = i32()
        check(lib().tb_b200_runner_position(self._h, C.byref(p)), "runner_position")
        return p.value

    @property
    def stream(self):
        s = vp()
        check(lib().tb_b200_runner_stream(self._h, C.byref(s)), "runner_stream")
        return s

    @property
    def launches_per_token(self):
        n = i32()
        check(lib().tb_b200_runner_launches_per_token(self._h, C.byref(n)), "runner_launches")
        return n.value

    def close(self):
        if getattr(self, "_h", None):
            lib().tb_b200_runner_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class TbmModel:
    """A .tbm container read into device memory (tb_b200_tbm_load)."""

    def __init__(self, path, stream=None):
        h = vp()
        check(lib().tb_b200_tbm_load(str(path).encode(), stream or cur_stream(), C.byref(h)),
              "tbm_load")
        self._h = h

    def config(self) -> TbmConfig:
        c = TbmConfig()
        check(lib().tb_b200_tbm_config(self._h, C.byref(c)), "tbm_config")
        return c

    def __len__(self):
        n = i32()
        check(lib().tb_b200_tbm_count(self._h, C.byref(n)), "tbm_count")
        return n.value

    def tensor(self, i):
        """(return code, TbmTensor) of tensor i: TB_OK, or TB_ERR_BAD_MAGIC
        for a tensor whose .tb header is not one."""
        t = TbmTensor()
        rc = lib().tb_b200_tbm_tensor(self._h, i, C.byref(t))
        return rc, t

    def find(self, name):
        i = i32()
        rc = lib().tb_b200_tbm_find(self._h, name.encode(), C.byref(i))
        return i.value if rc == 0 else -1

    def runner(self, attention=ATTN_REFERENCE, use_graph=True, max_layers=512):
        """A device runner over this model's tensors (borrowed: the model
        must stay open while the runner lives)."""
        layers = (RunnerLayer * max_layers)()
        d = RunnerDesc()
        check(lib().tb_b200_tbm_runner_desc(self._h, attention, 1 if use_graph else 0,
                                            C.byref(d), layers, max_layers), "tbm_runner_desc")
        return Runner.from_desc(d, d.vocab, keep=(layers, self))

    def close(self):
        if getattr(self, "_h", None):
            check(lib().tb_b200_tbm_free(self._h), "tbm_free")
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
