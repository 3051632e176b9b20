"""GPU parity at the reference configurations' full sizes.

Every op here runs once over the whole synthetic input of a full-size
configuration (Llama-70B prefill: 16384 rows; the bandwidth sweep's largest
points), generated on the device from a fixed seed.  Rows are independent,
so a seeded sample of rows (plus the first and the last) is checked against
the CPU oracle exactly as the smaller parity tests check whole tensors:
bit-exact for gathers, argmax, residual adds and RoPE at table positions,
1 bf16 ulp / 1e-5 row-relative otherwise (tests/parity.py).  Argmax is
checked on every row.
"""
import numpy as np
import pytest

import tb_b200 as T
import workloads as W
from oracle import oracle as O
from parity import assert_bf16, assert_bitexact, assert_f32, to_np

pytestmark = pytest.mark.gpu

SAMPLE = 192  # rows checked per full-size launch, besides the first and the last


@pytest.fixture(scope="module")
def dev(cuda):
    import torch
    torch.cuda.set_device(cuda)
    yield cuda
    torch.cuda.empty_cache()


def sample_rows(n, seed, k=SAMPLE):
    rng = np.random.default_rng(seed)
    pick = rng.choice(n, size=min(k, n), replace=False)
    return np.unique(np.concatenate([pick, [0, n - 1]])).astype(np.int64)


def randn(torch, dev, shape, seed, std=1.0, mean=0.0, dtype=None):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    t = torch.randn(shape, generator=g, device=dev) * std + mean
    return t if dtype is None else t.to(dtype)


def rows_of(t, idx):
    import torch
    return to_np(t[torch.from_numpy(idx).to(t.device)])


def test_llama70b_layer_chain_full_size(dev):
    """16384 tokens, hidden 8192, 64/8 heads x 128, intermediate 28672,
    theta 5e5, positions 0..16383, bf16: the fused chain in one launch."""
    import torch
    c = W.CONFIGS["70b"]
    bf = torch.bfloat16
    x = randn(torch, dev, (c.rows, c.hidden), 40, dtype=bf)
    res = randn(torch, dev, (c.rows, c.hidden), 41, dtype=bf)
    gamma = randn(torch, dev, (c.hidden,), 42, std=0.1, mean=1.0, dtype=bf)
    q = randn(torch, dev, (c.rows, c.n_q_heads, c.head_dim), 43, dtype=bf)
    k = randn(torch, dev, (c.rows, c.n_kv_heads, c.head_dim), 44, dtype=bf)
    gate = randn(torch, dev, (c.rows, c.intermediate), 45, dtype=bf)
    up = randn(torch, dev, (c.rows, c.intermediate), 46, dtype=bf)
    pos = torch.arange(c.rows, dtype=torch.int32, device=dev)
    idx = sample_rows(c.rows, 70)
    q0, k0 = rows_of(q, idx), rows_of(k, idx)  # RoPE works in place
    h, y, act = torch.empty_like(x), torch.empty_like(x), torch.empty_like(gate)
    table = T.rope_table(c.theta, c.head_dim, c.rows)
    T.layer_chain(T.make_chain(x, res, gamma, h, y, c.eps, q, k, pos, c.theta, table, gate, up,
                               act))
    torch.cuda.synchronize()
    assert T.check_status() == (0, 0)

    xs, rs = rows_of(x, idx), rows_of(res, idx)
    h_ref, y_ref = O.residual_rms_norm(xs, rs, to_np(gamma), c.eps, threads=8)
    assert_bitexact(rows_of(h, idx), h_ref, "70b h = x + residual")
    assert_bf16(rows_of(y, idx), y_ref, "70b RMSNorm y")
    q_ref, k_ref = O.rope(q0, k0, idx.astype(np.int32), c.theta, threads=8)
    assert_bitexact(rows_of(q, idx), q_ref, "70b RoPE q")
    assert_bitexact(rows_of(k, idx), k_ref, "70b RoPE k")
    a_ref = O.swiglu(rows_of(gate, idx), rows_of(up, idx), threads=8)
    assert_bf16(rows_of(act, idx), a_ref, "70b SwiGLU")


def test_llama70b_embedding_full_size(dev):
    """16384 ids U[0, 128256) from a 128256 x 8192 bf16 table (2.1 GB)."""
    import torch
    c = W.CONFIGS["70b"]
    table = randn(torch, dev, (c.vocab, c.hidden), 47, std=0.02, dtype=torch.bfloat16)
    g = torch.Generator(device=dev)
    g.manual_seed(48)
    ids = torch.randint(0, c.vocab, (c.rows,), generator=g, device=dev, dtype=torch.int32)
    out = T.embedding(ids, table)
    torch.cuda.synchronize()
    assert T.check_status() == (0, 0)
    idx = sample_rows(c.rows, 71, k=2048)
    ids_s = to_np(ids)[idx]
    assert_bitexact(rows_of(out, idx), O.embedding(ids_s, to_np(table), threads=8),
                    "70b embedding")


def test_sweep_softmax_and_argmax_128k_vocab_4096_rows(dev):
    """The sweep's widest point: 4096 rows of 128256 f32 logits N(0, 3)."""
    import torch
    rows, vocab = 4096, 128256
    x = randn(torch, dev, (rows, vocab), 49, std=3.0)
    y = T.softmax(x)
    am = T.argmax(x)
    torch.cuda.synchronize()
    assert T.check_status() == (0, 0)
    idx = sample_rows(rows, 72, k=48)
    xs = rows_of(x, idx)
    assert_f32(rows_of(y, idx), O.softmax(xs, threads=8), "softmax 4096 x 128256")
    assert_bitexact(to_np(am), O.argmax(to_np(x), threads=8), "argmax 4096 x 128256 (all rows)")


@pytest.mark.parametrize("rows,hidden,dtype", [(1 << 20, 2048, "bf16"), (1 << 18, 16384, "bf16"),
                                               (1 << 16, 16384, "f32")])
def test_sweep_residual_rms_norm_full_size(dev, rows, hidden, dtype):
    import torch
    dt = torch.bfloat16 if dtype == "bf16" else torch.float32
    x = randn(torch, dev, (rows, hidden), 50, dtype=dt)
    res = randn(torch, dev, (rows, hidden), 51, dtype=dt)
    gamma = randn(torch, dev, (hidden,), 52, std=0.1, mean=1.0, dtype=dt)
    h = torch.empty_like(x)
    _, y = T.residual_rms_norm(x, res, gamma, 1e-5, h_out=h)
    torch.cuda.synchronize()
    assert T.check_status() == (0, 0)
    idx = sample_rows(rows, 73)
    h_ref, y_ref = O.residual_rms_norm(rows_of(x, idx), rows_of(res, idx), to_np(gamma), 1e-5,
                                       threads=8)
    assert_bitexact(rows_of(h, idx), h_ref, f"h {rows}x{hidden}")
    if dtype == "bf16":
        assert_bf16(rows_of(y, idx), y_ref, f"y {rows}x{hidden}")
    else:
        assert_f32(rows_of(y, idx), y_ref, f"y {rows}x{hidden}")


@pytest.mark.parametrize("rows,inter,dtype", [(1 << 20, 2048, "bf16"), (1 << 18, 16384, "bf16"),
                                              (16384, 28672, "f32")])
def test_sweep_swiglu_full_size(dev, rows, inter, dtype):
    import torch
    dt = torch.bfloat16 if dtype == "bf16" else torch.float32
    gate = randn(torch, dev, (rows, inter), 53, dtype=dt)
    up = randn(torch, dev, (rows, inter), 54, dtype=dt)
    out = T.swiglu(gate, up)
    torch.cuda.synchronize()
    assert T.check_status() == (0, 0)
    idx = sample_rows(rows, 74)
    ref = O.swiglu(rows_of(gate, idx), rows_of(up, idx), threads=8)
    if dtype == "bf16":
        assert_bf16(rows_of(out, idx), ref, f"swiglu {rows}x{inter}")
    else:
        assert_f32(rows_of(out, idx), ref, f"swiglu {rows}x{inter}")
