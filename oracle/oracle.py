"""CPU oracle for the tensorbit-run row-op hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` use this module, and only as the checker or the timed CPU
reference; the shipped library never loads it.

It wraps ``oracle/liboracle.so`` (the C restatement in ``port.c`` plus the
row-batched drivers in ``rows.c``) and, when present, ``oracle/_ref/libtbref.so``
(the reference's own ``src/ops/*.c`` compiled unmodified by ``oracle/Makefile``).
Arrays are numpy; bf16 arrays are carried as ``np.uint16`` bit patterns.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libtbref.so")
PIN_SAMPLING_SO = os.path.join(HERE, "_ref", "libpinsampling.so")
PIN_DEQUANT_SO = os.path.join(HERE, "_ref", "libpindequant.so")

PORT, REF = 0, 1
F32, BF16 = 0, 2  # TbDtype codes (include/tensorbit/run/common.h:89-99)

_lib = None


def build(quiet: bool = True) -> None:
    """Compile liboracle.so (and _ref/ when the reference tree is present)."""
    out = subprocess.run(["make", "-C", HERE, "all"], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    if not quiet:
        print(out.stdout)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(PORT_SO):
            build()
        _lib = C.CDLL(PORT_SO)
        _declare(_lib)
        if os.path.exists(REF_SO):
            _lib.orc_load_ref(REF_SO.encode())
    return _lib


def ref_available() -> bool:
    return bool(lib().orc_ref_loaded())


def _declare(L: C.CDLL) -> None:
    vp, i64, i32, f32 = C.c_void_p, C.c_int64, C.c_int, C.c_float
    L.orc_load_ref.argtypes = [C.c_char_p]
    L.orc_rows_residual_rms_norm.argtypes = [i32, i32, i64, i64, vp, vp, vp, vp, vp, f32, i32]
    L.orc_rows_rms_norm.argtypes = [i32, i32, i64, i64, vp, vp, vp, f32, i32]
    L.orc_rows_residual_add.argtypes = [i32, i32, i64, i64, vp, vp, vp, i32]
    L.orc_rows_gelu.argtypes = [i32, i32, i64, i64, vp, vp, i32]
    L.orc_rows_silu.argtypes = [i32, i32, i64, i64, vp, vp, i32]
    L.orc_rows_swiglu.argtypes = [i32, i32, i64, i64, vp, vp, vp, i32]
    L.orc_rows_rope.argtypes = [i32, i32, i64, i32, i32, i32, vp, vp, vp, f32, i32]
    L.orc_rows_softmax.argtypes = [i32, i32, i64, i64, vp, vp, vp, i32]
    L.orc_rows_argmax.argtypes = [i32, i32, i64, i64, vp, vp, i32]
    L.orc_rows_embedding.argtypes = [i32, i32, i64, i64, vp, vp, vp, i32]
    L.orc_rms_norm_f32.argtypes = [C.c_size_t, vp, vp, vp, f32]
    L.orc_softmax_f32.argtypes = [C.c_size_t, vp, vp, vp]
    L.orc_argmax_f32.argtypes = [vp, i32]
    L.orc_uniforms.argtypes = [C.c_uint32, i64, vp]
    L.orc_rows_sample_temperature.argtypes = [i64, i64, vp, f32, vp, vp, i32]
    L.orc_dequant_f32.argtypes = [i32, C.c_size_t, vp, vp, C.c_size_t, C.c_uint32, vp]


# ---------------------------------------------------------------- helpers
def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _dt(a: np.ndarray) -> int:
    if a.dtype == np.float32:
        return F32
    if a.dtype == np.uint16:
        return BF16
    raise TypeError(f"oracle: unsupported dtype {a.dtype}")


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"oracle {what} failed with code {rc}")


def _c(a):
    return None if a is None else np.ascontiguousarray(a)


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bits (NaN kept quiet)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x0040).astype(np.uint16)
    return r


def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(a, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------- row ops
def residual_rms_norm(x, res, weight, eps, impl=PORT, threads=1):
    x, res, weight = _c(x), _c(res), _c(weight)
    rows, cols = x.shape
    h = np.empty_like(x)
    y = np.empty_like(x)
    _check(lib().orc_rows_residual_rms_norm(impl, _dt(x), rows, cols, _p(x), _p(res), _p(weight),
                                            _p(h), _p(y), eps, threads), "residual_rms_norm")
    return h, y


def rms_norm(x, weight, eps, impl=PORT, threads=1):
    x, weight = _c(x), _c(weight)
    rows, cols = x.shape
    y = np.empty_like(x)
    _check(lib().orc_rows_rms_norm(impl, _dt(x), rows, cols, _p(x), _p(weight), _p(y), eps,
                                   threads), "rms_norm")
    return y


def residual_add(x, res, impl=PORT, threads=1):
    x, res = _c(x), _c(res)
    rows, cols = x.shape
    y = np.empty_like(x)
    _check(lib().orc_rows_residual_add(impl, _dt(x), rows, cols, _p(x), _p(res), _p(y), threads),
           "residual_add")
    return y


def gelu(x, impl=PORT, threads=1):
    x = _c(x)
    rows, cols = x.shape
    y = np.empty_like(x)
    _check(lib().orc_rows_gelu(impl, _dt(x), rows, cols, _p(x), _p(y), threads), "gelu")
    return y


def silu(x, impl=PORT, threads=1):
    x = _c(x)
    rows, cols = x.shape
    y = np.empty_like(x)
    _check(lib().orc_rows_silu(impl, _dt(x), rows, cols, _p(x), _p(y), threads), "silu")
    return y


def swiglu(gate, up, impl=PORT, threads=1):
    gate, up = _c(gate), _c(up)
    rows, cols = gate.shape
    out = np.empty_like(gate)
    _check(lib().orc_rows_swiglu(impl, _dt(gate), rows, cols, _p(gate), _p(up), _p(out), threads),
           "swiglu")
    return out


def rope(q, k, positions, theta, impl=PORT, threads=1):
    """q [R, Hq, d], k [R, Hkv, d]; returns rotated copies."""
    q = np.array(q, copy=True, order="C")
    k = np.array(k, copy=True, order="C")
    pos = np.ascontiguousarray(positions, dtype=np.int32)
    rows, hq, d = q.shape
    hkv = k.shape[1]
    _check(lib().orc_rows_rope(impl, _dt(q), rows, hq, hkv, d, _p(q), _p(k), _p(pos), theta,
                               threads), "rope")
    return q, k


def softmax(x, mask=None, impl=PORT, threads=1):
    x, mask = _c(x), _c(mask)
    rows, cols = x.shape
    y = np.empty_like(x)
    _check(lib().orc_rows_softmax(impl, _dt(x), rows, cols, _p(x), _p(mask), _p(y), threads),
           "softmax")
    return y


def argmax(x, impl=PORT, threads=1):
    x = _c(x)
    rows, cols = x.shape
    out = np.empty(rows, dtype=np.int32)
    _check(lib().orc_rows_argmax(impl, _dt(x), rows, cols, _p(x), _p(out), threads), "argmax")
    return out


def embedding(ids, table, impl=PORT, threads=1):
    ids, table = np.ascontiguousarray(ids, dtype=np.int32), _c(table)
    dim = table.shape[1]
    y = np.empty((ids.shape[0], dim), dtype=table.dtype)
    _check(lib().orc_rows_embedding(impl, _dt(table), ids.shape[0], dim, _p(ids), _p(table),
                                    _p(y), threads), "embedding")
    return y


# ---------------------------------------------------------------- vectors
def rms_norm_vec(x, weight, eps):
    """The per-vector kernel itself (one call, one vector)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = None if weight is None else np.ascontiguousarray(weight, dtype=np.float32)
    y = np.empty_like(x)
    _check(lib().orc_rms_norm_f32(x.size, _p(x), _p(w), _p(y), eps), "rms_norm_f32")
    return y


def softmax_vec(x, mask=None):
    x = np.ascontiguousarray(x, dtype=np.float32)
    m = None if mask is None else np.ascontiguousarray(mask, dtype=np.float32)
    y = np.empty_like(x)
    _check(lib().orc_softmax_f32(x.size, _p(x), _p(m), _p(y)), "softmax_f32")
    return y


# ------------------------------------------------------- temperature sampling
def uniforms(seed: int, count: int) -> np.ndarray:
    """The first `count` generate_canonical<double, 53> values of
    std::mt19937(seed), as the reference's discrete_distribution draws them."""
    out = np.empty(count, dtype=np.float64)
    lib().orc_uniforms(seed & 0xFFFFFFFF, count, _p(out))
    return out


def sample_temperature(logits, temperature, u, threads=1):
    """sample_temperature (src/main.cpp:91-111) per row of f32 logits, the
    discrete_distribution draw taken at the given uniform u[row]."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    rows, cols = logits.shape
    u = np.ascontiguousarray(u, dtype=np.float64)
    out = np.empty(rows, dtype=np.int32)
    _check(lib().orc_rows_sample_temperature(rows, cols, _p(logits), temperature, _p(u), _p(out),
                                             threads), "sample_temperature")
    return out


def pin_available() -> bool:
    return os.path.exists(PIN_SAMPLING_SO)


def _pin():
    L = C.CDLL(PIN_SAMPLING_SO)
    L.pin_sample_temperature_rows.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_float,
                                              C.c_uint32, C.c_void_p]
    L.pin_uniforms.argtypes = [C.c_uint32, C.c_int64, C.c_void_p]
    return L


def pin_sample_temperature(logits, temperature, seed):
    """The same draws through libstdc++'s own mt19937 / discrete_distribution
    (oracle/_ref/libpinsampling.so), one per row in row order."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    rows, cols = logits.shape
    out = np.empty(rows, dtype=np.int32)
    _pin().pin_sample_temperature_rows(_p(logits), rows, cols, temperature, seed & 0xFFFFFFFF,
                                       _p(out))
    return out


def pin_uniforms(seed: int, count: int) -> np.ndarray:
    out = np.empty(count, dtype=np.float64)
    _pin().pin_uniforms(seed & 0xFFFFFFFF, count, _p(out))
    return out


# ----------------------------------------------------------- INT4/INT8 weights
INT8, INT4 = 7, 8  # TbDtype codes


def dequant(dtype: int, q, scales, group_size: int, n: int) -> np.ndarray:
    """Model::get_weight_fp32 (include/tensorbit/run/model.hpp:181-225) on n
    quantized weights `q` (uint8 bytes: INT4 packed two per byte, INT8 one)."""
    q = np.ascontiguousarray(q, dtype=np.uint8)
    scales = np.ascontiguousarray(scales, dtype=np.float32)
    out = np.empty(n, dtype=np.float32)
    _check(lib().orc_dequant_f32(dtype, n, _p(q), _p(scales), scales.size, group_size, _p(out)),
           "dequant")
    return out


def pin_dequant_available() -> bool:
    return os.path.exists(PIN_DEQUANT_SO)


def pin_dequant(dtype: int, q, scales, group_size: int, rows: int, cols: int) -> np.ndarray:
    """The reference's own Model::get_weight_fp32 on the same bytes
    (oracle/_ref/libpindequant.so)."""
    L = C.CDLL(PIN_DEQUANT_SO)
    L.pin_dequant_f32.argtypes = [C.c_int, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p,
                                  C.c_int64, C.c_uint32, C.c_void_p]
    q = np.ascontiguousarray(q, dtype=np.uint8)
    scales = np.ascontiguousarray(scales, dtype=np.float32)
    out = np.empty(rows * cols, dtype=np.float32)
    _check(L.pin_dequant_f32(dtype, rows, cols, _p(q), _p(scales), scales.size, group_size,
                             _p(out)), "pin_dequant")
    return out


# ------------------------------------------------------------- linear (GEMV)
def linear(x, w, mask=None, bias=None, nm_n=2, nm_m=4, impl=PORT):
    """y = W x (+ bias): tb_cpu_sparse_linear_f32 when `mask` is given, else
    tb_cpu_dense_linear_f32 (src/ops/linear.c:4-53); impl REF calls the
    reference's own functions in oracle/_ref/libtbref.so."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out_f, in_f = w.shape
    y = np.empty(out_f, dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    if impl == REF:
        L = C.CDLL(REF_SO)
        sp, dn = L.tb_cpu_sparse_linear_f32, L.tb_cpu_dense_linear_f32
    else:
        L = lib()
        sp, dn = L.orc_sparse_linear_f32, L.orc_dense_linear_f32
    if mask is not None:
        m = np.ascontiguousarray(mask, dtype=np.uint8)
        sp.argtypes = [C.c_size_t, C.c_size_t, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                       C.c_void_p, C.c_int, C.c_int]
        _check(sp(out_f, in_f, _p(x), _p(w), _p(m), _p(b), _p(y), nm_n, nm_m), "sparse_linear")
    else:
        dn.argtypes = [C.c_size_t, C.c_size_t, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
        _check(dn(out_f, in_f, _p(x), _p(w), _p(b), _p(y)), "dense_linear")
    return y


# ------------------------------------------------- decoder forward (runner)
PIN_RUNNER_SO = os.path.join(HERE, "_ref", "libpinrunner.so")
ATTN_REFERENCE, ATTN_STANDARD = 0, 1
PROJECTIONS = ("q", "k", "v", "o", "gate", "up", "down")
CFG_FIELDS = ("hidden", "n_heads", "n_kv_heads", "head_dim", "intermediate", "vocab", "max_seq",
              "layers")


class _Lin(C.Structure):
    _fields_ = [("w", C.c_void_p), ("mask", C.c_void_p), ("rows", C.c_int64),
                ("cols", C.c_int64)]


class _Layer(C.Structure):
    _fields_ = [(n, _Lin) for n in PROJECTIONS] + [("in_norm", C.c_void_p),
                                                   ("post_norm", C.c_void_p)]


class _Model(C.Structure):
    _fields_ = [("embed", C.c_void_p), ("final_norm", C.c_void_p), ("lm_head", C.c_void_p),
                ("layers", C.POINTER(_Layer))]


class _Cfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in CFG_FIELDS] + [("norm_eps", C.c_float),
                                                     ("rope_theta", C.c_float),
                                                     ("attention", C.c_int)]


def _runner_args(cfg: dict, model: dict):
    """ctypes views of a model dict: {"embed", "final_norm", "lm_head",
    "layers": [{"q": (w, mask or None), ..., "in_norm", "post_norm"}]} with
    f32 numpy weights; keeps the arrays alive in the returned tuple."""
    keep = []

    def arr(a, dt=np.float32):
        if a is None:
            return None
        a = np.ascontiguousarray(a, dtype=dt)
        keep.append(a)
        return a.ctypes.data

    layers = (_Layer * max(1, len(model["layers"])))()
    for i, ly in enumerate(model["layers"]):
        for n in PROJECTIONS:
            w, m = ly.get(n, (None, None))
            if w is not None:
                setattr(layers[i], n, _Lin(arr(w), arr(m, np.uint8), w.shape[0], w.shape[1]))
        layers[i].in_norm = arr(ly.get("in_norm"))
        layers[i].post_norm = arr(ly.get("post_norm"))
    m = _Model(arr(model["embed"]), arr(model.get("final_norm")), arr(model.get("lm_head")),
               layers)
    c = _Cfg(*[int(cfg[n]) for n in CFG_FIELDS], float(cfg.get("norm_eps", 1e-5)),
             float(cfg.get("rope_theta", 10000.0)), int(cfg.get("attention", ATTN_REFERENCE)))
    return c, m, (keep, layers)


def runner_run(cfg: dict, model: dict, tokens, impl=PORT) -> np.ndarray:
    """Logits [len(tokens), vocab] after each token of a fresh decoder
    (TransformerRunner::forward, include/tensorbit/run/ops.hpp:79-288):
    impl PORT is oracle/runner.c, REF the reference's own runner
    (oracle/_ref/libpinrunner.so)."""
    c, m, keep = _runner_args(cfg, model)
    toks = np.ascontiguousarray(tokens, dtype=np.int32)
    out = np.empty((toks.size, int(cfg["vocab"])), dtype=np.float32)
    if impl == REF:
        L = C.CDLL(PIN_RUNNER_SO)
        fn = L.pin_runner_run
    else:
        fn = lib().orc_runner_run
    fn.argtypes = [C.POINTER(_Cfg), C.POINTER(_Model), C.c_int, C.c_void_p, C.c_void_p]
    _check(fn(C.byref(c), C.byref(m), toks.size, _p(toks), _p(out)), "runner")
    del keep
    return out


def pin_runner_available() -> bool:
    return os.path.exists(PIN_RUNNER_SO)
