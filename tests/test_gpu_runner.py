"""GPU parity of the device decoder (tb_b200_runner_*, TransformerRunner
on the device) and of its attention step (tb_b200_decode_attention) with
the reference's TransformerRunner::forward
(include/tensorbit/run/ops.hpp:79-288).

The oracle is oracle/runner.c, bit-exact with the reference's own runner
over its CPU backend on the engine's mock model (tests/test_oracle.py); the
reference itself (oracle/_ref/libpinrunner.so) is compared too where it
travelled with the tree.  The device sums its GEMVs, norms and attention in
a different order from the reference's left-to-right loops, so each token's
logits are compared as a vector: max |g - c| <= TOL * max |c|."""
import numpy as np
import pytest

import tb_b200 as T
from oracle import oracle as O
from runner_models import mock, quantize

pytestmark = pytest.mark.gpu

# Relative tolerance on a token's logit vector.  The reordered f32 sums of
# two layers of GEMVs differ from the reference's by a few 1e-7 of the
# largest logit.
TOL = 2e-5


@pytest.fixture(scope="module")
def dev(cuda):
    import torch
    torch.cuda.set_device(cuda)
    return cuda


def run_device(cfg, model, tokens, attention=T.ATTN_REFERENCE, use_graph=True):
    r = T.Runner(cfg, model, attention=attention, use_graph=use_graph)
    out = []
    for t in tokens:
        r.forward(int(t))
        out.append(r.logits())
    r.close()
    return np.stack(out)


def assert_logits(got, want, tol=TOL):
    for t in range(want.shape[0]):
        err = np.abs(got[t] - want[t]).max()
        scale = np.abs(want[t]).max()
        assert err <= tol * scale, f"token {t}: max err {err:.3e} vs max |logit| {scale:.3e}"


def tokens(n, vocab, seed=5):
    return np.random.default_rng(seed).integers(0, vocab, n).astype(np.int32)


@pytest.mark.parametrize("use_graph", [True, False])
def test_mock_model_matches_reference(dev, use_graph):
    """The engine's mock model (tb-run --mock's shape), all 64 positions."""
    cfg, model = mock(seed=11)
    toks = tokens(64, cfg["vocab"])
    want = O.runner_run(cfg, model, toks)
    got = run_device(cfg, model, toks, use_graph=use_graph)
    assert_logits(got, want)
    if O.pin_runner_available():
        assert_logits(got, O.runner_run(cfg, model, toks, O.REF))


def test_graph_and_eager_are_identical(dev):
    cfg, model = mock(seed=13, masks="rand", norms="rand")
    toks = tokens(20, cfg["vocab"])
    a = run_device(cfg, model, toks, use_graph=True)
    b = run_device(cfg, model, toks, use_graph=False)
    assert np.array_equal(a, b)


@pytest.mark.parametrize("masks,norms", [("rand", "rand"), ("none", "rand"), ("mixed", "ones")])
def test_random_masks_and_dense_projections(dev, masks, norms):
    cfg, model = mock(seed=17, masks=masks, norms=norms, layers=3)
    toks = tokens(32, cfg["vocab"])
    assert_logits(run_device(cfg, model, toks), O.runner_run(cfg, model, toks))


@pytest.mark.parametrize("attention", [T.ATTN_REFERENCE, T.ATTN_STANDARD])
@pytest.mark.parametrize("heads,kv", [(8, 8), (8, 2), (16, 4)])
def test_attention_layouts_and_gqa(dev, attention, heads, kv):
    cfg, model = mock(seed=19, hidden=512, inter=1024, heads=heads, kv=kv, vocab=300,
                      max_seq=48, masks="rand", norms="rand")
    cfg["attention"] = attention
    toks = tokens(48, cfg["vocab"])
    assert_logits(run_device(cfg, model, toks, attention=attention), O.runner_run(cfg, model, toks))


def test_tied_lm_head_and_wide_vocab(dev):
    """No lm_head tensor: the embedding table is the head (ops.hpp:269-273);
    vocab above hidden (the device norms cover hidden floats)."""
    cfg, model = mock(seed=23, vocab=1000, tied=True, masks="rand")
    toks = tokens(16, cfg["vocab"])
    assert_logits(run_device(cfg, model, toks), O.runner_run(cfg, model, toks))


@pytest.mark.parametrize("bits,group_size", [(8, 128), (4, 64), (4, 0)])
def test_quantized_projections(dev, bits, group_size):
    """INT8 / INT4 projections are dequantised once on the device to the
    values Model::get_weight_fp32 gives (model.hpp:181-225)."""
    cfg, model = mock(seed=29, masks="rand")
    qmodel = dict(model, layers=[])
    ref_layers = []
    for ly in model["layers"]:
        ql, rl = dict(ly), dict(ly)
        for n in ("q", "k", "v", "o", "gate", "up", "down"):
            w, m = ly[n]
            data, scales = quantize(w, bits, group_size)
            dt = T.INT8 if bits == 8 else T.INT4
            ql[n] = (T.QuantWeight(data, dt, w.shape[0], w.shape[1], scales, group_size), m)
            rl[n] = (O.dequant(dt, data, scales, group_size, w.size).reshape(w.shape), m)
        qmodel["layers"].append(ql)
        ref_layers.append(rl)
    toks = tokens(12, cfg["vocab"])
    want = O.runner_run(cfg, dict(model, layers=ref_layers), toks)
    assert_logits(run_device(cfg, qmodel, toks), want)


def test_device_resident_weights_are_borrowed(dev):
    import torch
    cfg, model = mock(seed=31, masks="rand")
    dmodel = dict(model, embed=torch.from_numpy(model["embed"]).to(dev))
    dmodel["layers"] = [dict(ly, q=(torch.from_numpy(ly["q"][0]).to(dev),
                                    torch.from_numpy(ly["q"][1]).to(dev)))
                        for ly in model["layers"]]
    toks = tokens(8, cfg["vocab"])
    assert_logits(run_device(cfg, dmodel, toks), O.runner_run(cfg, model, toks))


def test_reset_replays_the_sequence_and_errors_queue_nothing(dev):
    cfg, model = mock(seed=37, max_seq=8)
    toks = tokens(8, cfg["vocab"])
    r = T.Runner(cfg, model)
    first = []
    for t in toks:
        r.forward(int(t))
        first.append(r.logits())
    assert r.position == 8
    with pytest.raises(T.TbError):  # cache full: max_seq positions used
        r.forward(0)
    r.reset()
    assert r.position == 0
    with pytest.raises(T.TbError):
        r.forward(cfg["vocab"])
    with pytest.raises(T.TbError):
        r.forward(-1)
    again = []
    for t in toks:
        r.forward(int(t))
        again.append(r.logits())
    assert np.array_equal(np.stack(first), np.stack(again))
    assert T.check_status(r.stream) == (0, 0)
    r.close()


@pytest.mark.parametrize("mode", [T.ATTN_REFERENCE, T.ATTN_STANDARD])
@pytest.mark.parametrize("heads,kv,d,pos", [(32, 32, 128, 2047), (8, 2, 64, 300), (4, 4, 32, 0),
                                            (64, 8, 128, 4095)])
def test_decode_attention_kernel(dev, mode, heads, kv, d, pos):
    """The attention step alone against its float64 definition, up to a
    4096-position cache (Llama-7B and 70B head shapes)."""
    import torch
    rng = np.random.default_rng(41)
    max_seq = max(pos + 1, 64)
    kvd = kv * d
    kc = rng.standard_normal((max_seq, kvd)).astype(np.float32)
    vc = rng.standard_normal((max_seq, kvd)).astype(np.float32)
    q = rng.standard_normal(heads * d).astype(np.float32)
    k = rng.standard_normal(kvd).astype(np.float32)
    v = rng.standard_normal(kvd).astype(np.float32)
    g = {n: torch.from_numpy(a).to(dev) for n, a in dict(kc=kc, vc=vc, q=q, k=k, v=v).items()}
    p = torch.tensor([pos], dtype=torch.int32, device=dev)
    out = T.decode_attention(g["q"], g["k"], g["v"], g["kc"], g["vc"], p, heads, kv, mode)
    torch.cuda.synchronize()
    kc[pos], vc[pos] = k, v
    cur = pos + 1
    want = np.zeros((heads, d))
    for r in range(heads):
        h, last = (r // cur, r % cur) if mode == T.ATTN_REFERENCE else (r, pos)
        gk = h // (heads // kv)
        s = kc[:last + 1, gk * d:(gk + 1) * d].astype(np.float64) @ q[h * d:(h + 1) * d] / np.sqrt(d)
        e = np.exp(s - s.max())
        want[r] = (e / e.sum()) @ vc[:last + 1, gk * d:(gk + 1) * d]
    got = out.cpu().numpy().reshape(heads, d)
    np.testing.assert_allclose(got, want, rtol=0, atol=2e-5 * np.abs(want).max())
    # the token's k and v were appended at row pos
    assert np.array_equal(g["kc"][pos].cpu().numpy(), k)
    assert np.array_equal(g["vc"][pos].cpu().numpy(), v)


@pytest.mark.parametrize("which", ["v", "v_cache", "k"])
def test_decode_attention_unaligned_operand(dev, which):
    """k, v and the caches are read as float4 only when every one of them is
    16-byte aligned: a slice of a packed buffer one float off (for example v
    inside a fused qkv vector) takes the scalar path and gives the same
    attention as aligned copies of the same values."""
    import torch
    rng = np.random.default_rng(43)
    heads, kv, d, pos = 8, 2, 64, 37
    max_seq, kvd = 64, kv * d
    vals = {n: rng.standard_normal(s).astype(np.float32)
            for n, s in dict(q=heads * d, k=kvd, v=kvd, k_cache=max_seq * kvd,
                             v_cache=max_seq * kvd).items()}

    def run(off):
        g = {}
        for n, a in vals.items():
            pad = 1 if n == off else 0
            buf = torch.zeros(a.size + pad, dtype=torch.float32, device=dev)
            buf[pad:] = torch.from_numpy(a).to(dev)
            g[n] = buf[pad:]
        g["k_cache"] = g["k_cache"].view(max_seq, kvd)
        g["v_cache"] = g["v_cache"].view(max_seq, kvd)
        p = torch.tensor([pos], dtype=torch.int32, device=dev)
        out = T.decode_attention(g["q"], g["k"], g["v"], g["k_cache"], g["v_cache"], p, heads, kv,
                                 T.ATTN_STANDARD)
        torch.cuda.synchronize()
        return out.cpu().numpy(), g

    want, _ = run(None)
    got, g = run(which)
    assert T.check_status() == (0, 0)
    np.testing.assert_allclose(got, want, rtol=0, atol=2e-6 * np.abs(want).max())
    assert np.array_equal(g["v_cache"][pos].cpu().numpy(), vals["v"])


@pytest.mark.parametrize("inter,masks", [(16384, "rand"), (8192, "none"), (8192, "rand")])
def test_rows_split_over_warps(dev, inter, masks):
    """Few output rows with long rows (a down projection of 128 rows over
    8192 or 16384 inputs): the fused GEMV splits each row pair over 4 or 8
    warps and adds their parts in a fixed order."""
    cfg, model = mock(seed=43, hidden=128, heads=4, kv=4, inter=inter, layers=1, vocab=100,
                      max_seq=16, masks=masks, norms="rand")
    toks = tokens(12, cfg["vocab"])
    a = run_device(cfg, model, toks)
    assert_logits(a, O.runner_run(cfg, model, toks))
    assert np.array_equal(a, run_device(cfg, model, toks, use_graph=False))


def test_long_rows_split_over_ctas(dev):
    """Standard attention past 512 keys: each head's row is split over
    several CTAs whose partial max, sum and weighted values the last one
    combines (in a fixed order: graph and eager replays agree bit for
    bit)."""
    cfg, model = mock(seed=47, layers=2, max_seq=1024, masks="rand", norms="rand")
    cfg["attention"] = T.ATTN_STANDARD
    toks = tokens(700, cfg["vocab"], seed=9)
    want = O.runner_run(cfg, model, toks)
    a = run_device(cfg, model, toks, attention=T.ATTN_STANDARD)
    assert_logits(a, want)
    b = run_device(cfg, model, toks[:600], attention=T.ATTN_STANDARD, use_graph=False)
    assert np.array_equal(a[:600], b)


def quantized_model(cfg, model, bits, group_size, names=("q", "k", "v", "o", "gate", "up", "down")):
    """The model with the named projections quantized (.tbm INT8/INT4
    layout), and the oracle's model over their dequantised weights."""
    dt = T.INT8 if bits == 8 else T.INT4
    qlayers, rlayers = [], []
    for ly in model["layers"]:
        ql, rl = dict(ly), dict(ly)
        for n in names:
            w, m = ly[n]
            data, scales = quantize(w, bits, group_size)
            ql[n] = (T.QuantWeight(data, dt, w.shape[0], w.shape[1], scales, group_size), m)
            rl[n] = (O.dequant(dt, data, scales, group_size, w.size).reshape(w.shape), m)
        qlayers.append(ql)
        rlayers.append(rl)
    return dict(model, layers=qlayers), dict(model, layers=rlayers)


@pytest.mark.parametrize("bits,group_size", [(8, 64), (8, 0), (4, 128), (4, 32), (4, 0), (4, 96)])
def test_unmasked_quantized_projections_stay_quantized(dev, bits, group_size):
    """Unmasked INT8/INT4 projections are read as bytes by the fused GEMV,
    each weight expanded to (float)q * scale in registers (group sizes 0 and
    powers of two from 8); other group sizes (96) are dequantised at load."""
    cfg, model = mock(seed=53, masks="none", norms="rand")
    qmodel, rmodel = quantized_model(cfg, model, bits, group_size)
    toks = tokens(24, cfg["vocab"])
    a = run_device(cfg, qmodel, toks)
    assert_logits(a, O.runner_run(cfg, rmodel, toks))
    assert np.array_equal(a, run_device(cfg, qmodel, toks, use_graph=False))


def test_quantized_and_f32_projections_mixed(dev):
    """Only q and down quantized: the layer's groups no longer share one
    layout, so each projection is its own launch."""
    cfg, model = mock(seed=59, masks="none", layers=2)
    qmodel, rmodel = quantized_model(cfg, model, 4, 64, names=("q", "down"))
    toks = tokens(16, cfg["vocab"])
    assert_logits(run_device(cfg, qmodel, toks), O.runner_run(cfg, rmodel, toks))


def test_quantized_long_rows_split(dev):
    """INT4 down projection of 128 rows over 8192 inputs: rows split over
    several warps."""
    cfg, model = mock(seed=61, hidden=128, heads=4, kv=4, inter=8192, layers=1, vocab=100,
                      max_seq=16, masks="none", norms="rand")
    qmodel, rmodel = quantized_model(cfg, model, 4, 128)
    toks = tokens(10, cfg["vocab"])
    assert_logits(run_device(cfg, qmodel, toks), O.runner_run(cfg, rmodel, toks))
