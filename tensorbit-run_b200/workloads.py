"""Synthetic workloads with the shapes and value distributions of the
reference engine's layer-op configurations.

There is no dataset on this path: inputs are seeded draws.  Each config has
a seed base; tensor k of a config uses seed base + k (numpy PCG64), so the
same inputs can be regenerated on any host for the CPU oracle and the GPU.

  mock     the engine's mock model (tb-run --mock): hidden 256, intermediate
           1024, 4 heads x 64, vocab 100, 64 tokens, fp32
  7b       Llama-7B prefill, 4096 tokens: hidden 4096, 32 heads x 128,
           intermediate 11008, vocab 32000, theta 1e4
  decode   batch 256 x 1 token at the 7B shape, positions U[0, 4096), bf16
  70b      Llama-3-70B prefill, 16384 tokens: hidden 8192, 64/8 heads x 128,
           intermediate 28672, vocab 128256, theta 5e5, bf16
Distributions: activations N(0,1); RMSNorm gamma 1 + N(0, 0.1); eps 1e-5;
embedding table N(0, 0.02); ids U[0, vocab); logits N(0, 2) (mock) or
N(0, 3).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class Config:
    name: str
    rows: int
    hidden: int
    intermediate: int
    n_q_heads: int
    n_kv_heads: int
    head_dim: int
    vocab: int
    theta: float
    logit_std: float
    seed: int
    positions: str = "arange"  # or "uniform4096"
    eps: float = 1e-5


CONFIGS = {
    "mock": Config("mock", 64, 256, 1024, 4, 4, 64, 100, 1e4, 2.0, 1000),
    "7b": Config("7b", 4096, 4096, 11008, 32, 32, 128, 32000, 1e4, 3.0, 2000),
    "decode": Config("decode", 256, 4096, 11008, 32, 32, 128, 32000, 1e4, 3.0, 3000,
                     positions="uniform4096"),
    "70b": Config("70b", 16384, 8192, 28672, 64, 8, 128, 128256, 5e5, 3.0, 4000),
}


def rng(cfg: Config, k: int) -> np.random.Generator:
    return np.random.default_rng(cfg.seed + k)


def normal(cfg: Config, k: int, shape, std=1.0, mean=0.0) -> np.ndarray:
    a = rng(cfg, k).standard_normal(size=shape, dtype=np.float32)
    if std != 1.0:
        a *= np.float32(std)
    if mean != 0.0:
        a += np.float32(mean)
    return a


def positions(cfg: Config, rows: int | None = None) -> np.ndarray:
    rows = cfg.rows if rows is None else rows
    if cfg.positions == "arange":
        return np.arange(rows, dtype=np.int32)
    return rng(cfg, 90).integers(0, 4096, size=rows, dtype=np.int32)


def layer_inputs(cfg: Config, rows: int | None = None) -> dict:
    """f32 inputs of one layer's row ops (tensor k = seed offset k)."""
    r = cfg.rows if rows is None else rows
    return {
        "x": normal(cfg, 0, (r, cfg.hidden)),
        "res": normal(cfg, 1, (r, cfg.hidden)),
        "gamma": normal(cfg, 2, (cfg.hidden,), std=0.1, mean=1.0),
        "q": normal(cfg, 3, (r, cfg.n_q_heads, cfg.head_dim)),
        "k": normal(cfg, 4, (r, cfg.n_kv_heads, cfg.head_dim)),
        "gate": normal(cfg, 5, (r, cfg.intermediate)),
        "up": normal(cfg, 6, (r, cfg.intermediate)),
        "pos": positions(cfg, r),
    }


def embedding_inputs(cfg: Config, rows: int | None = None) -> dict:
    r = cfg.rows if rows is None else rows
    return {
        "table": normal(cfg, 7, (cfg.vocab, cfg.hidden), std=0.02),
        "ids": rng(cfg, 8).integers(0, cfg.vocab, size=r, dtype=np.int32),
    }


def logits(cfg: Config, rows: int | None = None, cols: int | None = None) -> np.ndarray:
    r = cfg.rows if rows is None else rows
    c = cfg.vocab if cols is None else cols
    return normal(cfg, 9, (r, c), std=cfg.logit_std)


# Algorithmic HBM bytes per op (s = bytes per element): each input read once,
# each output written once.
def bytes_res_rms(rows, hidden, s):
    return 4 * rows * hidden * s + hidden * s


def bytes_rope(rows, hq, hkv, d, s):
    return 2 * rows * (hq + hkv) * d * s + 4 * rows


def bytes_swiglu(rows, inter, s):
    return 3 * rows * inter * s


def bytes_unary(rows, inter, s):
    return 2 * rows * inter * s


def bytes_embedding(rows, hidden, s):
    return 2 * rows * hidden * s + 4 * rows


def bytes_softmax(rows, vocab, s):
    return 2 * rows * vocab * s


def bytes_argmax(rows, vocab, s):
    return rows * vocab * s + 4 * rows
