"""Parity criteria shared by the GPU tests.

- Integer/index/byte ops (embedding gather, argmax, residual add, the h
  output of residual+RMSNorm, RoPE at table positions): bit-exact.
- f32 ops: row-wise max-norm relative error  max|g - c| / max|c| <= 1e-5
  per row (elementwise relative error is meaningless where the result
  cancels to ~0, e.g. GELU for x < -3 or a RoPE output near 0); the
  elementwise max-abs error is reported with it.
- bf16 ops: every element within 1 bf16 ulp of bf16_rne(oracle_f32(widened
  inputs)), the oracle's bf16 mode -- or, where the f32 result cancels to
  ~0 (GELU's 1 + tanhf for x < -3), within the f32 bound 1e-5 * max|row|
  that the f32 criterion already allows before rounding.
- elementwise ops are judged in rows of 1024 consecutive elements.
NaN must match NaN.
"""
import numpy as np

F32_ROW_REL = 1e-5
BF16_ULPS = 1


def to_np(t):
    import torch
    t = t.detach()
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    return t.cpu().numpy()


def from_np(a, device):
    import torch
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).to(device)
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def assert_bitexact(g, c, what=""):
    g, c = np.asarray(g), np.asarray(c)
    assert g.shape == c.shape, (what, g.shape, c.shape)
    same = g.view(np.uint8).reshape(-1) == c.view(np.uint8).reshape(-1)
    if not same.all():
        flat_g, flat_c = g.reshape(-1), c.reshape(-1)
        i = int(np.argmin(same.reshape(flat_g.size, -1).all(axis=1)))
        raise AssertionError(f"{what}: not bit-exact, first difference at {i}: "
                             f"{flat_g[i]!r} vs {flat_c[i]!r}")


def rowwise_rel(g, c):
    g = np.asarray(g, np.float64).reshape(g.shape[0], -1)
    c = np.asarray(c, np.float64).reshape(c.shape[0], -1)
    nan_g, nan_c = np.isnan(g), np.isnan(c)
    assert (nan_g == nan_c).all(), "NaN positions differ"
    g = np.where(nan_g, 0, g)
    c = np.where(nan_c, 0, c)
    err = np.abs(g - c).max(axis=1)
    scale = np.abs(c).max(axis=1)
    rel = np.where(scale > 0, err / np.where(scale > 0, scale, 1), np.where(err > 0, np.inf, 0))
    return rel, float(np.abs(g - c).max()) if g.size else 0.0


def assert_f32(g, c, what="", tol=F32_ROW_REL):
    g, c = np.asarray(g), np.asarray(c)
    assert g.shape == c.shape, (what, g.shape, c.shape)
    if g.size == 0:
        return 0.0, 0.0
    rel, maxabs = rowwise_rel(g, c)
    worst = float(rel.max())
    assert worst <= tol, f"{what}: row-wise relative error {worst:.3e} > {tol} (max abs {maxabs:.3e})"
    return worst, maxabs


def bf16_ordinal(u):
    u = np.asarray(u, np.uint16).astype(np.int32)
    return np.where(u & 0x8000, -(u & 0x7FFF), u)


def _bf16_f32(u):
    return (np.asarray(u, np.uint16).astype(np.uint32) << 16).view(np.float32)


def assert_bf16(g, c, what="", ulps=BF16_ULPS, row_floor=F32_ROW_REL):
    g, c = np.asarray(g, np.uint16), np.asarray(c, np.uint16)
    assert g.shape == c.shape, (what, g.shape, c.shape)
    if g.size == 0:
        return 0
    nan_g = (g & 0x7FFF) > 0x7F80
    nan_c = (c & 0x7FFF) > 0x7F80
    assert (nan_g == nan_c).all(), f"{what}: NaN positions differ"
    d = np.abs(bf16_ordinal(g) - bf16_ordinal(c))
    gf = _bf16_f32(g).astype(np.float64).reshape(g.shape[0], -1)
    cf = _bf16_f32(c).astype(np.float64).reshape(c.shape[0], -1)
    with np.errstate(invalid="ignore"):
        scale = np.nanmax(np.where(np.isinf(cf), 0, np.abs(cf)), axis=1, keepdims=True)
        near = np.abs(gf - cf) <= row_floor * scale
    bad = (d.reshape(gf.shape) > ulps) & ~near & ~nan_c.reshape(gf.shape)
    assert not bad.any(), (f"{what}: {int(bad.sum())} elements beyond {ulps} bf16 ulp "
                           f"(worst {int(d.reshape(gf.shape)[bad].max())} ulps)")
    return int(d[~nan_c].max()) if (~nan_c).any() else 0


def blocks(a, width=1024):
    """Flatten and cut into rows of `width` (zero-padded tail)."""
    a = np.asarray(a).reshape(-1)
    pad = (-a.size) % width
    if pad:
        a = np.concatenate([a, np.zeros(pad, a.dtype)])
    return a.reshape(-1, width) if a.size else a.reshape(0, width)
