""".tbm containers for the device-loader tests, and the reference's own
container code (oracle/_ref/libpintbm.so, built from src/model.c) to write
and read them.

- ``write_ref`` writes an f32 model through the reference's writer,
  tb_tbm_create (src/model.c:747-860), under the names TransformerRunner
  looks up (include/tensorbit/run/ops.hpp:61-116, 259-276).  Every
  projection gets mask bytes (all-ones 2:4 groups for a dense one): the
  reference runner always reads a projection's mask (Model::get_mask), and
  without mask bytes it would read whatever follows the weights.
- ``write_quant`` writes INT4 / INT8 projections, which the reference's
  writer cannot (tb_dtype_size(INT4) is 0), laid out as its loader reads
  them (docs/TBM_FORMAT.md; src/model.c:280-341 for the index keys and
  718-739 for the scales after the quantized weights).
- ``RefTbm`` opens a file with the reference's loader, tb_model_load_tbm,
  and returns each tensor's descriptor and its zero-copy views.
"""
import ctypes as C
import json
import os
import struct

import numpy as np

from oracle import oracle as O

PIN_TBM_SO = os.path.join(os.path.dirname(O.PORT_SO), "_ref", "libpintbm.so")

F32, INT8, INT4 = 0, 7, 8
MAGIC, VERSION, HEADER = 0x31304254, 1, 4096


class RefConfig(C.Structure):  # TbModelConfig (include/tensorbit/run/model.h:34-46)
    _fields_ = [("architecture", C.c_char * 64)] + [
        (n, C.c_int) for n in ("hidden_size", "num_heads", "num_kv_heads", "intermediate_size",
                               "vocab_size", "max_seq_len", "num_layers")] + [
        ("norm_eps", C.c_float), ("rope_theta", C.c_float), ("head_dim", C.c_int)]


class _Layer(C.Structure):
    _fields_ = [("name", C.c_char_p), ("rows", C.c_uint64), ("cols", C.c_uint64),
                ("nm_n", C.c_int), ("nm_m", C.c_int), ("dtype", C.c_int), ("w", C.c_void_p),
                ("w_bytes", C.c_uint64), ("mask", C.c_void_p), ("mask_bytes", C.c_uint64)]


class _Info(C.Structure):
    _fields_ = [("name", C.c_char * 128), ("shape", C.c_uint64 * 2), ("dtype", C.c_int),
                ("nm_n", C.c_uint32), ("nm_m", C.c_uint32), ("num_weights", C.c_uint64),
                ("num_mask_bytes", C.c_uint64), ("scale_count", C.c_uint64),
                ("group_size", C.c_uint32), ("w", C.c_void_p), ("m", C.c_void_p),
                ("s", C.c_void_p), ("rc_w", C.c_int), ("rc_m", C.c_int), ("rc_s", C.c_int)]


def available():
    return os.path.exists(PIN_TBM_SO)


def _lib():
    L = C.CDLL(PIN_TBM_SO)
    L.pin_tbm_create.argtypes = [C.c_char_p, C.POINTER(RefConfig), C.c_int, C.POINTER(_Layer)]
    L.pin_tbm_open.argtypes = [C.c_char_p, C.POINTER(C.c_void_p)]
    L.pin_tbm_config.argtypes = [C.c_void_p, C.POINTER(RefConfig)]
    L.pin_tbm_count.argtypes = [C.c_void_p]
    L.pin_tbm_info.argtypes = [C.c_void_p, C.c_int, C.POINTER(_Info)]
    L.pin_tbm_close.argtypes = [C.c_void_p]
    L.pin_tbm_runner.argtypes = [C.c_char_p, C.c_int, C.c_void_p, C.c_void_p, C.c_int]
    return L


def ref_config(cfg, arch="llama"):
    return RefConfig(arch.encode(), cfg["hidden"], cfg["n_heads"], cfg["n_kv_heads"],
                     cfg["intermediate"], cfg["vocab"], cfg["max_seq"], cfg["layers"],
                     cfg.get("norm_eps", 1e-5), cfg.get("rope_theta", 1e4),
                     cfg["hidden"] // cfg["n_heads"])


NAMES = dict(q="self_attn.q_proj", k="self_attn.k_proj", v="self_attn.v_proj",
             o="self_attn.o_proj", gate="mlp.gate_proj", up="mlp.up_proj", down="mlp.down_proj")


def tensors_of(cfg, model, dense_masks=True):
    """[(name, f32 array [rows, cols], mask bytes or None)] in the names the
    reference runner looks up."""
    out = [("model.embed_tokens.weight", model["embed"], None)]
    for l, ly in enumerate(model["layers"]):
        p = f"model.layers.{l}."
        for n, comp in NAMES.items():
            w, m = ly[n][0], (ly[n][1] if len(ly[n]) > 1 else None)
            if m is None and dense_masks and not isinstance(w, tuple):
                m = np.full((w.shape[0], w.shape[1] // 4), 0x0F, np.uint8)
            out.append((p + comp + ".weight", w, m))
        out.append((p + "input_layernorm.weight", ly["in_norm"], None))
        out.append((p + "post_attention_layernorm.weight", ly["post_norm"], None))
    out.append(("model.norm.weight", model["final_norm"], None))
    if model.get("lm_head") is not None:
        out.append(("lm_head.weight", model["lm_head"], None))
    return out


def write_ref(path, cfg, model):
    """The f32 model through the reference's tb_tbm_create."""
    keep, layers = [], []
    for name, w, m in tensors_of(cfg, model):
        w = np.ascontiguousarray(w, np.float32)
        keep.append(w)
        rows, cols = (w.shape[0], w.shape[1]) if w.ndim == 2 else (w.shape[0], 0)
        lay = _Layer(name.encode(), rows, cols, 2 if m is not None else 0,
                     4 if m is not None else 0, F32, w.ctypes.data, w.nbytes, None, 0)
        if m is not None:
            m = np.ascontiguousarray(m, np.uint8)
            keep.append(m)
            lay.mask, lay.mask_bytes = m.ctypes.data, m.nbytes
        layers.append(lay)
    arr = (_Layer * len(layers))(*layers)
    rc = _lib().pin_tbm_create(str(path).encode(), C.byref(ref_config(cfg)), len(layers), arr)
    if rc != 0:
        raise RuntimeError(f"tb_tbm_create: {rc}")


def _header(nm_n, nm_m, num_weights, num_mask_bytes, w_bytes, magic=MAGIC):
    h = struct.pack("<IIIIQQQQB", magic, VERSION, nm_n, nm_m, num_weights, num_mask_bytes,
                    HEADER, HEADER + w_bytes, 0)
    return h + b"\0" * (HEADER - len(h))


def write_quant(path, cfg, entries, bad_magic=()):
    """entries: [(name, kind, payload)] with kind "f32" (array), "int4" /
    "int8" ((packed bytes, scales, rows, cols, group_size)); optional mask
    bytes as a fourth element.  Tensors named in bad_magic get a wrong
    header magic."""
    idx, blob = [], bytearray()
    for e in entries:
        name, kind, payload = e[0], e[1], e[2]
        mask = e[3] if len(e) > 3 and e[3] is not None else None
        off = len(blob)
        if kind == "f32":
            w = np.ascontiguousarray(payload, np.float32)
            data, nw = w.tobytes(), w.size
            shape = [w.shape[0], w.shape[1] if w.ndim == 2 else 0]
            rec = dict(dtype="fp32")
        else:
            q, sc, rows, cols, gs = payload
            data = np.ascontiguousarray(q, np.uint8).tobytes() + \
                np.ascontiguousarray(sc, np.float32).tobytes()
            nw, shape = rows * cols, [rows, cols]
            rec = dict(dtype=kind, scale_count=int(np.size(sc)), group_size=int(gs))
        mb = b"" if mask is None else np.ascontiguousarray(mask, np.uint8).tobytes()
        nm = (2, 4) if mask is not None else (0, 0)
        blob += _header(nm[0], nm[1], nw, len(mb), len(data),
                        magic=(0xDEADBEEF if name in bad_magic else MAGIC))
        blob += data + mb
        blob += b"\0" * (-len(blob) % 64)
        idx.append(dict(name=name, offset=off, shape=shape, nm_n=nm[0], nm_m=nm[1],
                        num_weights=nw, num_mask_bytes=len(mb), **rec))
    index = dict(architecture="llama",
                 config=dict(hidden_size=cfg["hidden"], num_heads=cfg["n_heads"],
                             num_kv_heads=cfg["n_kv_heads"],
                             intermediate_size=cfg["intermediate"], vocab_size=cfg["vocab"],
                             num_layers=cfg["layers"], max_seq_len=cfg["max_seq"],
                             norm_eps=cfg.get("norm_eps", 1e-5),
                             rope_theta=cfg.get("rope_theta", 1e4)),
                 tensors=idx)
    js = json.dumps(index).encode()
    with open(path, "wb") as f:
        f.write(bytes(blob) + js + struct.pack("<I", len(js)))


class RefTbm:
    """A file opened by the reference's tb_model_load_tbm."""

    def __init__(self, path):
        self.L = _lib()
        self.h = C.c_void_p()
        self.rc = self.L.pin_tbm_open(str(path).encode(), C.byref(self.h))

    def config(self):
        c = RefConfig()
        self.L.pin_tbm_config(self.h, C.byref(c))
        return c

    def __len__(self):
        return self.L.pin_tbm_count(self.h)

    def info(self, i):
        x = _Info()
        self.L.pin_tbm_info(self.h, i, C.byref(x))
        return x

    def close(self):
        if self.h:
            self.L.pin_tbm_close(self.h)
            self.h = None


def ref_runner(path, tokens, vocab):
    """The reference's TransformerRunner over the model loaded from `path`."""
    toks = np.ascontiguousarray(tokens, np.int32)
    out = np.empty((toks.size, vocab), np.float32)
    rc = _lib().pin_tbm_runner(str(path).encode(), toks.size, toks.ctypes.data, out.ctypes.data,
                               vocab)
    if rc != 0:
        raise RuntimeError(f"reference runner over {path}: {rc}")
    return out
