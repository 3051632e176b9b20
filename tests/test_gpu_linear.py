"""GPU parity of the linear layers (tb_b200_sparse_linear /
tb_b200_dense_linear) with the reference's tb_cpu_sparse_linear_f32 and
tb_cpu_dense_linear_f32 (src/ops/linear.c:4-53), through the oracle (bit-
exact with the reference's own functions, tests/test_oracle.py).

The reference accumulates each output left to right; the device sums in a
different order, so outputs are compared with the f32 row criterion of
tests/parity.py over the output vector (max |g - c| / max |c| <= 1e-5)."""
import numpy as np
import pytest

import tb_b200 as T
from oracle import oracle as O
from parity import assert_f32, from_np, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev(cuda):
    import torch
    torch.cuda.set_device(cuda)
    return cuda


def nm_mask(rng, out_f, in_f, n, m):
    groups = in_f // m
    bits = np.zeros((out_f, groups), np.uint8)
    for _ in range(n):
        bits |= (1 << rng.integers(0, m, (out_f, groups))).astype(np.uint8)
    return bits


# Llama-7B decode projections (q/k/v/o 4096 x 4096, gate/up 11008 x 4096,
# down 4096 x 11008), the mock model's, and odd shapes.
SHAPES = [(4096, 4096), (11008, 4096), (4096, 11008), (256, 256), (1024, 256), (100, 37), (3, 5),
          (1, 4096)]


@pytest.mark.parametrize("out_f,in_f", SHAPES)
@pytest.mark.parametrize("sparse", [True, False])
@pytest.mark.parametrize("with_bias", [True, False])
def test_linear_matches_reference(dev, out_f, in_f, sparse, with_bias):
    rng = np.random.default_rng(out_f * 7 + in_f)
    x = rng.standard_normal(in_f).astype(np.float32)
    w = (rng.standard_normal((out_f, in_f)) * 0.02).astype(np.float32)
    b = rng.standard_normal(out_f).astype(np.float32) if with_bias else None
    mask = nm_mask(rng, out_f, in_f, 2, 4) if sparse else None
    got = to_np(T.linear(from_np(x, dev), from_np(w, dev),
                         None if mask is None else from_np(mask, dev),
                         None if b is None else from_np(b, dev)))
    want = O.linear(x, w, mask, b)
    assert_f32(got[None, :], want[None, :], f"linear {out_f}x{in_f} sparse={sparse}")


@pytest.mark.parametrize("n,m", [(1, 8), (3, 4), (1, 2), (4, 16)])
def test_sparse_linear_other_n_m(dev, n, m):
    """Other N:M (M = 16 uses one byte per group, as the reference does:
    weights whose bit is past 7 are never kept)."""
    out_f, in_f = 300, 1000
    rng = np.random.default_rng(n * 10 + m)
    x = rng.standard_normal(in_f).astype(np.float32)
    w = rng.standard_normal((out_f, in_f)).astype(np.float32)
    mask = nm_mask(rng, out_f, in_f, min(n, 8), min(m, 8))
    mask = np.ascontiguousarray(mask[:, :in_f // m]) if m > 8 else mask
    got = to_np(T.linear(from_np(x, dev), from_np(w, dev), from_np(mask, dev), None, n, m))
    assert_f32(got[None, :], O.linear(x, w, mask, None, n, m)[None, :], f"{n}:{m}")


def test_linear_argument_errors(dev):
    import torch
    L = T.lib()
    v = torch.zeros(16, device=dev)
    m = torch.zeros(16, dtype=torch.uint8, device=dev)
    assert L.tb_b200_sparse_linear(4, 4, T.ptr(v), T.ptr(v), T.ptr(m), None, T.ptr(v), 2, 1, None) == 8
    assert L.tb_b200_sparse_linear(4, 4, T.ptr(v), T.ptr(v), None, None, T.ptr(v), 2, 4, None) == 8
    assert L.tb_b200_dense_linear(4, 4, None, T.ptr(v), None, T.ptr(v), None) == 8


# ------------------------------------------- packed 2:4 form (k_sparse24.cu)
def mask_with_kept(rng, out_f, in_f, kept_choices):
    """Mask bytes whose groups keep a random number of weights from
    kept_choices (bits in random positions; bits 4-7 random noise)."""
    groups = in_f // 4
    out = np.zeros((out_f, groups), np.uint8)
    ks = rng.choice(kept_choices, (out_f, groups))
    for k in set(kept_choices):
        sel = ks == k
        perm = np.argsort(rng.random((int(sel.sum()), 4)), axis=1)[:, :k]
        bits = np.zeros(int(sel.sum()), np.uint8)
        for c in range(k):
            bits |= (1 << perm[:, c]).astype(np.uint8)
        out[sel] = bits
    return out | (rng.integers(0, 16, out.shape).astype(np.uint8) << 4)


@pytest.mark.parametrize("out_f,in_f", [(4096, 4096), (11008, 4096), (4096, 11008), (256, 256),
                                        (3, 8), (101, 72)])
@pytest.mark.parametrize("with_bias", [True, False])
def test_packed_2_4_linear_matches_reference(dev, out_f, in_f, with_bias):
    """Packed kept values + 2-bit indices give the reference's masked sum
    (groups keeping 0, 1 or 2 weights; high mask bits ignored as the
    reference ignores them)."""
    rng = np.random.default_rng(out_f + 3 * in_f)
    x = rng.standard_normal(in_f).astype(np.float32)
    w = (rng.standard_normal((out_f, in_f)) * 0.02).astype(np.float32)
    mask = mask_with_kept(rng, out_f, in_f, [2, 2, 2, 1, 0])
    b = rng.standard_normal(out_f).astype(np.float32) if with_bias else None
    vals, idx, ok = T.sparse24_pack(from_np(w, dev), from_np(mask, dev))
    assert ok
    got = to_np(T.sparse24_linear(from_np(x, dev), vals, idx, in_f,
                                  None if b is None else from_np(b, dev)))
    want = O.linear(x, w, mask, b)
    assert_f32(got[None, :], want[None, :], f"packed {out_f}x{in_f}")


def test_packed_2_4_detects_groups_keeping_three(dev):
    rng = np.random.default_rng(9)
    w = rng.standard_normal((64, 256)).astype(np.float32)
    mask = np.full((64, 64), 0x3, np.uint8)
    assert T.sparse24_pack(from_np(w, dev), from_np(mask, dev))[2]
    mask[17, 5] = 0x7
    assert not T.sparse24_pack(from_np(w, dev), from_np(mask, dev))[2]


def test_packed_2_4_rejects_odd_group_count(dev):
    import torch
    L = T.lib()
    v = torch.zeros(64, device=dev)
    m = torch.zeros(64, dtype=torch.uint8, device=dev)
    assert L.tb_b200_sparse24_linear(4, 12, T.ptr(v), T.ptr(v), T.ptr(m), None, T.ptr(v), None) == 9
