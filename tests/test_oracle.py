"""The CPU oracle, pinned to the reference.

1. The reference's own known-answer tests for this path, restated:
   tests/test_norm.c:23-57 (RMSNorm) and tests/test_softmax.c:33-68.
2. Golden checksums made by running the reference's unmodified kernels
   (tests/golden/make_golden.py): the restatement must reproduce them
   bit-for-bit.
3. Where the reference build (oracle/_ref) is present, the restatement and
   the reference agree bit-for-bit on fresh seeded inputs, for f32 and bf16.
4. Edge semantics of argmax (src/main.cpp:79-89) and softmax.
"""
import hashlib
import importlib.util
import json
import math
import os

import numpy as np
import pytest

from oracle import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))


def _golden_module():
    spec = importlib.util.spec_from_file_location(
        "make_golden", os.path.join(HERE, "golden", "make_golden.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


# ---------------------------------------------------------------- 1. KATs
def test_ref_kat_rms_norm_unit_weight():
    # tests/test_norm.c:23-40
    x = np.array([1, 2, 3, 4], np.float32)
    y = O.rms_norm_vec(x, np.ones(4, np.float32), 1e-6)
    rms = math.sqrt((1 + 4 + 9 + 16) / 4.0 + 1e-6)
    np.testing.assert_allclose(y, x / rms, atol=1e-4)


def test_ref_kat_rms_norm_weighted():
    # tests/test_norm.c:43-57
    y = O.rms_norm_vec(np.full(4, 2, np.float32), np.array([0.5, 1, 1.5, 2], np.float32), 0.0)
    np.testing.assert_allclose(y, [0.5, 1.0, 1.5, 2.0], atol=1e-4)


def test_ref_kat_softmax_basic():
    # tests/test_softmax.c:33-44
    y = O.softmax_vec(np.array([1, 2, 3], np.float32))
    assert abs(float(y.sum()) - 1.0) <= 1e-4
    assert y[2] > y[1] > y[0]


def test_ref_kat_softmax_uniform():
    # tests/test_softmax.c:47-56
    np.testing.assert_allclose(O.softmax_vec(np.full(4, 5, np.float32)), 0.25, atol=1e-4)


def test_ref_kat_softmax_mask():
    # tests/test_softmax.c:59-68
    y = O.softmax_vec(np.array([1, 2, 3], np.float32), np.array([0, 0, -100], np.float32))
    assert abs(float(y[2])) <= 1e-3
    assert y[1] > y[0]


# ------------------------------------------------------------ 2. golden
def test_golden_checksums_reproduced_by_port():
    meta = json.load(open(os.path.join(HERE, "golden", "golden.json")))
    mg = _golden_module()
    names = set()
    for name, fn in mg.cases():
        res = fn(O.PORT)
        for k, v in res.items():
            want = meta["cases"][name][k]
            assert list(v.shape) == want["shape"], (name, k)
            got = hashlib.sha256(np.ascontiguousarray(v).tobytes()).hexdigest()
            assert got == want["sha256"], f"{name}.{k}: port differs from the reference"
        names.add(name)
    assert names == set(meta["cases"]), "golden cases and generator out of sync"


def test_golden_rows_match_checksummed_outputs():
    rows = np.load(os.path.join(HERE, "golden", "golden_rows.npz"))
    mg = _golden_module()
    for name, fn in mg.cases():
        for k, v in fn(O.PORT).items():
            flat = v.reshape(v.shape[0], -1) if v.ndim > 1 else v.reshape(1, -1)
            np.testing.assert_array_equal(rows[f"{name}.{k}"], flat[[0, -1], :1024])


# ------------------------------------------------- 3. port vs reference
needs_ref = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built here")


def _same(a, b):
    return np.array_equal(np.asarray(a).view(np.uint8), np.asarray(b).view(np.uint8))


@needs_ref
@pytest.mark.parametrize("rows,cols", [(7, 4096), (3, 16384), (5, 100), (2, 1), (1, 8192)])
@pytest.mark.parametrize("bf16", [False, True])
def test_port_equals_reference_rowops(rows, cols, bf16):
    rng = np.random.default_rng(rows * 1000 + cols)
    cv = O.f32_to_bf16 if bf16 else (lambda a: a)
    x = cv(rng.standard_normal((rows, cols), dtype=np.float32))
    r = cv(rng.standard_normal((rows, cols), dtype=np.float32))
    w = cv((1 + 0.1 * rng.standard_normal(cols)).astype(np.float32))
    for a, b in zip(O.residual_rms_norm(x, r, w, 1e-5, O.PORT),
                    O.residual_rms_norm(x, r, w, 1e-5, O.REF)):
        assert _same(a, b)
    assert _same(O.rms_norm(x, w, 1e-6, O.PORT), O.rms_norm(x, w, 1e-6, O.REF))
    assert _same(O.gelu(x, O.PORT), O.gelu(x, O.REF))
    assert _same(O.silu(x, O.PORT), O.silu(x, O.REF))
    assert _same(O.swiglu(x, r, O.PORT), O.swiglu(x, r, O.REF))
    assert _same(O.residual_add(x, r, O.PORT), O.residual_add(x, r, O.REF))
    xs = cv(3 * rng.standard_normal((rows, cols), dtype=np.float32))
    assert _same(O.softmax(xs, None, O.PORT), O.softmax(xs, None, O.REF))
    assert _same(O.softmax(xs, r, O.PORT), O.softmax(xs, r, O.REF))


@needs_ref
@pytest.mark.parametrize("hq,hkv,d,theta", [(4, 4, 64, 1e4), (32, 32, 128, 1e4),
                                            (64, 8, 128, 5e5), (3, 1, 6, 1e4)])
def test_port_equals_reference_rope(hq, hkv, d, theta):
    rng = np.random.default_rng(hq * d)
    q = rng.standard_normal((9, hq, d), dtype=np.float32)
    k = rng.standard_normal((9, hkv, d), dtype=np.float32)
    pos = rng.integers(0, 20000, 9).astype(np.int32)
    for a, b in zip(O.rope(q, k, pos, theta, O.PORT), O.rope(q, k, pos, theta, O.REF)):
        assert _same(a, b)


@needs_ref
def test_port_equals_reference_embedding():
    rng = np.random.default_rng(5)
    t = rng.standard_normal((1000, 48), dtype=np.float32)
    ids = rng.integers(0, 1000, 333).astype(np.int32)
    assert _same(O.embedding(ids, t, O.PORT), O.embedding(ids, t, O.REF))


def test_threaded_rows_equal_single_thread():
    rng = np.random.default_rng(11)
    x = rng.standard_normal((37, 512), dtype=np.float32)
    assert _same(O.softmax(x, None, O.PORT, 1), O.softmax(x, None, O.PORT, 4))
    h1, y1 = O.residual_rms_norm(x, x, None, 1e-5, O.PORT, 1)
    h4, y4 = O.residual_rms_norm(x, x, None, 1e-5, O.PORT, 4)
    assert _same(y1, y4) and _same(h1, h4)


# ------------------------------------------------------- 4. edge cases
def test_argmax_semantics():
    nan, inf = np.float32("nan"), np.float32("inf")
    cases = [
        ([1, 3, 3, 2], 1),            # first maximum wins
        ([nan, 5, 7], 0),             # NaN at index 0 is never beaten
        ([1, nan, 0.5], 0),           # NaN never wins
        ([-inf, -inf], 0),            # nothing exceeds -inf
        ([-inf, nan, -inf], 0),
        ([-0.0, 0.0, -1], 0),         # +0 is not greater than -0
        ([-5, -inf, inf, inf], 2),
        ([2.0], 0),
    ]
    for vals, want in cases:
        got = O.argmax(np.array([vals], np.float32))[0]
        assert got == want, (vals, got)


def test_softmax_degenerate_rows_keep_exponentials():
    # softmax.c:24-29: a NaN or zero sum leaves y = exp(v - max) unnormalised.
    nan = np.float32("nan")
    y = O.softmax(np.array([[0.0, nan, 1.0]], np.float32))
    assert np.isnan(y[0, 1]) and y[0, 2] == 1.0 and y[0, 0] == np.float32(math.exp(-1.0))
    y = O.softmax(np.full((1, 3), -np.inf, np.float32))
    assert np.isnan(y).all()


def test_bf16_round_to_nearest_even():
    vals = np.array([1.0, 1.00390625, 1.01171875, 1.005859375, -2.5, 3.0e38, 1e-40],
                    np.float32)
    b = O.f32_to_bf16(vals)
    back = O.bf16_to_f32(b)
    # ties go to even: 1 + 2^-8 -> 1.0, 1 + 3*2^-8 -> 1 + 2^-6
    assert back[1] == 1.0 and back[2] == np.float32(1.015625)
    assert back[0] == 1.0 and back[4] == -2.5
    assert np.isnan(O.bf16_to_f32(O.f32_to_bf16(np.array([np.nan], np.float32))))[0]


# ------------------------------------------------------ temperature sampling
def test_mt19937_known_answer():
    """The C++ standard's check for mt19937: the 10000th output of a
    default-seeded (5489) engine is 4123659995."""
    import ctypes as C
    L = O.lib()
    L.orc_mt_seed.argtypes = [C.c_void_p, C.c_uint32]
    L.orc_mt_next.argtypes = [C.c_void_p]
    L.orc_mt_next.restype = C.c_uint32
    st = (C.c_uint8 * (624 * 4 + 8))()
    L.orc_mt_seed(st, 5489)
    for _ in range(9999):
        L.orc_mt_next(st)
    assert L.orc_mt_next(st) == 4123659995


def _sampling_rows():
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((64, 1000)) * 3).astype(np.float32)
    x[1, 0] = np.nan                 # the reference's max stays NaN
    x[2, 500] = np.nan               # a NaN weight
    x[3, 7] = np.inf                 # max = +inf: inf - inf
    x[4, :] = -np.inf                # every weight NaN
    x[5, 100:] = -np.inf             # zero weights
    x[6, :] = 2.5                    # equal weights: cp = (i + 1) / n
    x[7, :] = np.float32(1e30)       # one huge logit and the rest
    x[7, 3] = np.float32(-1e30)
    return x


@pytest.mark.skipif(not O.pin_available(), reason="libstdc++ pin not built (no reference tree)")
@pytest.mark.parametrize("temperature", [0.7, 1.0, 2.5, 1e-4, 1e4, 0.0, -1.0])
def test_sampling_restatement_matches_libstdcxx(temperature):
    """Oracle draws (restated discrete_distribution at the canonical u of its
    own mt19937) equal libstdc++'s own mt19937 + discrete_distribution."""
    x = _sampling_rows()
    u = O.uniforms(99, x.shape[0])
    assert np.array_equal(O.sample_temperature(x, temperature, u, threads=4),
                          O.pin_sample_temperature(x, temperature, 99))
    rng = np.random.default_rng(6)
    big = (rng.standard_normal((32, 32000)) * 3).astype(np.float32)
    assert np.array_equal(O.sample_temperature(big, temperature, O.uniforms(3, 32), threads=4),
                          O.pin_sample_temperature(big, temperature, 3))


@pytest.mark.skipif(not O.pin_available(), reason="libstdc++ pin not built (no reference tree)")
def test_canonical_draws_match_libstdcxx():
    for seed in (0, 1, 5489, 2**32 - 1):
        a, b = O.uniforms(seed, 5000), O.pin_uniforms(seed, 5000)
        assert np.array_equal(a.view(np.uint64), b.view(np.uint64))
        assert (a >= 0).all() and (a < 1).all()


def test_sampling_special_rows():
    """Rows whose weights hold a NaN draw index 0 (lower_bound over a NaN
    table); one logit draws 0 without a table; equal weights follow u."""
    x = _sampling_rows()
    u = np.full(x.shape[0], 0.5)
    got = O.sample_temperature(x, 1.0, u)
    assert got[1] == 0 and got[2] == 0 and got[3] == 0 and got[4] == 0
    assert 0 <= got[5] < 100
    assert got[6] == 499  # cp[i] = (i + 1) / 1000: first cp >= 0.5
    one = O.sample_temperature(np.array([[3.0]], np.float32), 1.0, np.array([0.9]))
    assert one[0] == 0


# ------------------------------------------------------ INT4 / INT8 weights
def _quant_case(dtype, rows, cols, group_size, seed):
    rng = np.random.default_rng(seed)
    n = rows * cols
    nbytes = (n + 1) // 2 if dtype == O.INT4 else n
    q = rng.integers(0, 256, nbytes, dtype=np.uint8)
    gs = group_size if group_size > 0 else n
    ngroups = (n + gs - 1) // gs
    scales = (rng.standard_normal(ngroups) * 0.01).astype(np.float32)
    return q, scales


@pytest.mark.skipif(not O.pin_dequant_available(), reason="reference build absent")
@pytest.mark.parametrize("dtype", [7, 8])
@pytest.mark.parametrize("rows,cols,group_size,drop", [(64, 256, 64, 0), (33, 101, 32, 0),
                                                       (7, 9, 0, 0), (16, 128, 128, 5),
                                                       (3, 5, 7, 0)])
def test_dequant_restatement_matches_reference(dtype, rows, cols, group_size, drop):
    """Bit-exact against the reference's own Model::get_weight_fp32; `drop`
    scales fewer than groups exercise the 1.0 default of missing scales."""
    q, scales = _quant_case(dtype, rows, cols, group_size, rows * cols + dtype)
    if drop:
        scales = scales[:-drop]
    n = rows * cols
    want = O.pin_dequant(dtype, q, scales, group_size, rows, cols)
    got = O.dequant(dtype, q, scales, group_size, n)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


# ------------------------------------------------------------- linear (GEMV)
def nm_mask(rng, out_f, in_f, n, m):
    """One byte per M-group with exactly n of the low m bits set."""
    groups = in_f // m
    bits = np.zeros((out_f, groups), np.uint8)
    for k in range(n):
        pick = rng.integers(0, m, (out_f, groups))
        bits |= (1 << pick).astype(np.uint8)
    return bits


@pytest.mark.skipif(not O.ref_available(), reason="reference build absent")
@pytest.mark.parametrize("out_f,in_f,n,m,with_bias", [(256, 1024, 2, 4, True), (100, 37, 2, 4, False),
                                                      (64, 4096, 1, 8, True), (33, 64, 3, 4, False)])
def test_linear_restatement_matches_reference(out_f, in_f, n, m, with_bias):
    rng = np.random.default_rng(out_f + in_f)
    x = rng.standard_normal(in_f).astype(np.float32)
    w = rng.standard_normal((out_f, in_f)).astype(np.float32)
    b = rng.standard_normal(out_f).astype(np.float32) if with_bias else None
    mask = nm_mask(rng, out_f, in_f, n, m)
    for msk in (mask, None):
        got = O.linear(x, w, msk, b, n, m, O.PORT)
        want = O.linear(x, w, msk, b, n, m, O.REF)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


# ------------------------------------------------- decoder forward (runner)
needs_pin_runner = pytest.mark.skipif(not O.pin_runner_available(),
                                      reason="reference runner (oracle/_ref) not built")


@needs_pin_runner
@pytest.mark.parametrize("masks,norms,tokens", [("mock", "ones", 64), ("rand", "rand", 24)])
def test_runner_restatement_matches_reference(masks, norms, tokens):
    """The reference's own TransformerRunner (ops.hpp:79-288 over its CPU
    backend) on the engine's mock shape: the restatement's logits after
    every token equal it bit for bit."""
    from runner_models import mock
    cfg, model = mock(seed=11, masks=masks, norms=norms)
    toks = np.random.default_rng(3).integers(0, cfg["vocab"], tokens).astype(np.int32)
    a = O.runner_run(cfg, model, toks, O.PORT)
    b = O.runner_run(cfg, model, toks, O.REF)
    assert np.array_equal(a, b)
    assert np.isfinite(a).all() and np.abs(a).max() > 0


@needs_pin_runner
def test_runner_dense_projections_match_reference_all_ones_masks():
    """A dense projection is the reference's 2:4 path with every mask bit
    set (all weights kept in order); the two differ only by FMA
    contraction in the inner loop."""
    from runner_models import mock
    cfg, model = mock(seed=12, masks="none", layers=1)
    toks = np.arange(10, dtype=np.int32)
    a = O.runner_run(cfg, model, toks, O.PORT)
    b = O.runner_run(cfg, model, toks, O.REF)
    assert np.abs(a - b).max() <= 1e-6 * np.abs(b).max()


def _attention_rows_np(q, kc, vc, pos, n_heads, n_kv, d, mode):
    """Float64 decode attention over a cache [pos+1, n_kv*d]."""
    cur = pos + 1
    out = np.zeros((n_heads, d))
    for r in range(n_heads):
        h, last = (r // cur, r % cur) if mode == O.ATTN_REFERENCE else (r, pos)
        g = h // (n_heads // n_kv)
        keys = kc[:last + 1, g * d:(g + 1) * d].astype(np.float64)
        vals = vc[:last + 1, g * d:(g + 1) * d].astype(np.float64)
        s = keys @ q[h * d:(h + 1) * d].astype(np.float64) / math.sqrt(d)
        p = np.exp(s - s.max())
        out[r] = (p / p.sum()) @ vals
    return out.reshape(-1)


@pytest.mark.parametrize("mode", [O.ATTN_REFERENCE, O.ATTN_STANDARD])
@pytest.mark.parametrize("heads,kv", [(8, 8), (8, 2)])
def test_runner_attention_rows_follow_their_definition(mode, heads, kv):
    """One layer with dense q/k/v, an identity output projection and lm
    head, no MLP and no norm weights: the logits after token t are
    rms_norm(x + attn) with x = rms_norm(embed[token]), so the attention
    rows (both layouts, MHA and GQA) can be replayed in float64 from their
    definition: softmax(q_h . k_j / sqrt(d)) over keys 0 .. last of kv head
    h / (heads / kv), weighted over v."""
    rng = np.random.default_rng(4)
    d, hidden = 16, 8 * 16
    kvd = kv * d
    cfg = dict(hidden=hidden, n_heads=heads, n_kv_heads=kv, head_dim=d, intermediate=0,
               vocab=hidden, max_seq=16, layers=1, norm_eps=1e-6, rope_theta=10000.0,
               attention=mode)
    wq = rng.standard_normal((heads * d, hidden)).astype(np.float32) * 0.3
    wk = rng.standard_normal((kvd, hidden)).astype(np.float32) * 0.3
    wv = rng.standard_normal((kvd, hidden)).astype(np.float32) * 0.3
    eye = np.eye(hidden, dtype=np.float32)
    embed = rng.standard_normal((hidden, hidden)).astype(np.float32)
    layer = dict(q=(wq, None), k=(wk, None), v=(wv, None), o=(eye, None))
    model = dict(embed=embed, final_norm=None, lm_head=eye, layers=[layer])
    toks = rng.integers(0, hidden, 9).astype(np.int32)
    got = O.runner_run(cfg, model, toks)
    kc = np.zeros((16, kvd), np.float32)
    vc = np.zeros((16, kvd), np.float32)
    for t, tok in enumerate(toks):
        x = O.rms_norm_vec(embed[tok], None, 1e-6)
        q, k = O.rope((wq @ x).reshape(1, heads, d), (wk @ x).reshape(1, kv, d),
                      np.array([t], np.int32), 10000.0)
        kc[t], vc[t] = k.reshape(-1), wv @ x
        att = _attention_rows_np(q.reshape(-1), kc, vc, t, heads, kv, d, mode)
        h = x.astype(np.float64) + att
        want = h / np.sqrt(((h * h).sum() + 1e-6) / hidden)  # src/ops/norm.c:8-13
        np.testing.assert_allclose(got[t], want, rtol=0, atol=2e-5 * np.abs(want).max())
