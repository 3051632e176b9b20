"""Seeded decoder models for the runner tests (the engine's mock model and
variants of it).

The reference's mock (src/main.cpp:117-300, what ``tb-run --mock`` builds):
hidden 256, intermediate 1024, 2 layers, vocab 100, 8 heads = 8 KV heads of
32, max_seq 64, every projection 2:4 with mask byte 0b0011, weights
U(-0.01, 0.01), norm weights 1, eps 1e-6, theta 10000.  ``mock`` builds that
shape from a numpy seed, with options for random 2:4 patterns, dense
projections, random norm weights, GQA and quantized projections.
"""
import numpy as np

PATTERNS_2_4 = np.array([0x3, 0x5, 0x6, 0x9, 0xA, 0xC], np.uint8)


def mock(seed=0, hidden=256, inter=1024, layers=2, vocab=100, heads=8, kv=8, max_seq=64,
         masks="mock", norms="ones", head_dim=None, tied=False):
    """(cfg, model) in the oracle's dict format: f32 numpy weights, uint8
    masks (None for dense)."""
    rng = np.random.default_rng(seed)
    d = head_dim or hidden // heads

    def w(r, c):
        return ((rng.random((r, c), dtype=np.float32) - 0.5) * 0.02).astype(np.float32)

    def mk(r, c):
        if masks == "none":
            return None
        if masks == "mock":
            return np.full((r, c // 4), 0x3, np.uint8)
        if masks == "mixed":  # some groups keep three or four weights
            return np.array([0x3, 0x7, 0xF, 0x5], np.uint8)[rng.integers(0, 4, (r, c // 4))]
        return PATTERNS_2_4[rng.integers(0, PATTERNS_2_4.size, (r, c // 4))]

    def nv():
        if norms == "ones":
            return np.ones(hidden, np.float32)
        return (1 + 0.1 * rng.standard_normal(hidden)).astype(np.float32)

    shapes = dict(q=(heads * d, hidden), k=(kv * d, hidden), v=(kv * d, hidden),
                  o=(hidden, heads * d), gate=(inter, hidden), up=(inter, hidden),
                  down=(hidden, inter))
    lys = []
    for _ in range(layers):
        ly = {n: (w(r, c), mk(r, c)) for n, (r, c) in shapes.items()}
        ly["in_norm"] = nv()
        ly["post_norm"] = nv()
        lys.append(ly)
    embed = w(vocab, hidden)
    model = dict(embed=embed, final_norm=nv(), lm_head=None if tied else w(vocab, hidden),
                 layers=lys)
    cfg = dict(hidden=hidden, n_heads=heads, n_kv_heads=kv, head_dim=d, intermediate=inter,
               vocab=vocab, max_seq=max_seq, layers=layers, norm_eps=1e-6, rope_theta=10000.0)
    return cfg, model


def quantize(w, bits, group_size):
    """Symmetric per-group quantization of an f32 [rows, cols] matrix to the
    .tbm INT8 / INT4 layout: (packed bytes, scales).  INT4 packs element i
    in the low nibble of byte i // 2 when i is even, the high nibble when
    odd (include/tensorbit/run/model.hpp:196-203)."""
    flat = w.reshape(-1)
    n = flat.size
    gs = group_size or n
    groups = (n + gs - 1) // gs
    qmax = 127 if bits == 8 else 7
    scales = np.empty(groups, np.float32)
    q = np.empty(n, np.int8)
    for g in range(groups):
        seg = flat[g * gs:(g + 1) * gs]
        s = np.float32(max(np.abs(seg).max(), 1e-12) / qmax)
        scales[g] = s
        q[g * gs:(g + 1) * gs] = np.clip(np.rint(seg / s), -qmax - 1, qmax).astype(np.int8)
    if bits == 8:
        return q.view(np.uint8).copy(), scales
    nib = (q.astype(np.int16) & 0xF).astype(np.uint8)
    if n % 2:
        nib = np.concatenate([nib, np.zeros(1, np.uint8)])
    packed = (nib[0::2] | (nib[1::2] << 4)).astype(np.uint8)
    return packed, scales
