""".tbm containers read into device memory (tb_b200_tbm_*), against the
reference's own container code (oracle/_ref/libpintbm.so: tb_tbm_create,
tb_model_load_tbm and its views, src/model.c:482-860; TransformerRunner over
the loaded file, include/tensorbit/run/ops.hpp:79-288).

For every tensor: the index entry (name, shape, dtype, N:M, counts, group
size) equals the reference loader's descriptor, and the device bytes of the
weights, mask and scales equal the bytes of the reference's zero-copy views,
bit for bit.  The runner made from the loaded file gives the same logits as
the device runner made from the same weights in host memory (bit for bit:
the same device code), and matches the reference runner over the file
within the runner tolerance (the device sums in a different order).
"""
import ctypes as C

import numpy as np
import pytest

import tb_b200 as T
import tbm_files as F
from oracle import oracle as O
from runner_models import mock, quantize

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not F.available(), reason="oracle/_ref/libpintbm.so not built")]

TOL = 2e-5  # as the runner tests: max |g - c| <= TOL * max |c| per token


@pytest.fixture(scope="module")
def dev(cuda):
    import torch
    torch.cuda.set_device(cuda)
    return cuda


def device_bytes(addr, n):
    out = np.empty(n, np.uint8)
    if n:
        T.check(T.lib().tb_b200_memcpy_d2h(out.ctypes.data, C.c_void_p(addr), n, None), "d2h")
        T.check(T.lib().tb_b200_stream_sync(None), "sync")
    return out


def host_bytes(addr, n):
    return np.frombuffer(C.string_at(addr, n), np.uint8) if n else np.empty(0, np.uint8)


def compare_with_reference(path):
    """Every tensor of `path`: the device loader against the reference's."""
    ref = F.RefTbm(path)
    assert ref.rc == 0
    m = T.TbmModel(path)
    rc, dc = ref.config(), m.config()
    for f, _ in F.RefConfig._fields_:
        assert getattr(rc, f) == getattr(dc, f), f"config {f}"
    assert len(m) == len(ref)
    for i in range(len(ref)):
        info = ref.info(i)
        code, t = m.tensor(i)
        assert t.name == info.name
        assert (t.shape[0], t.shape[1]) == (info.shape[0], info.shape[1])
        for f in ("dtype", "nm_n", "nm_m", "num_weights", "num_mask_bytes", "scale_count",
                  "group_size"):
            assert getattr(t, f) == getattr(info, f), f"{info.name}: {f}"
        assert code == info.rc_w, info.name
        if info.rc_w != 0:
            continue
        assert np.array_equal(device_bytes(t.weights, t.weight_bytes),
                              host_bytes(info.w, t.weight_bytes)), f"{info.name}: weights"
        if t.num_mask_bytes:
            assert info.rc_m == 0
            assert np.array_equal(device_bytes(t.mask, t.num_mask_bytes),
                                  host_bytes(info.m, t.num_mask_bytes)), f"{info.name}: mask"
        if t.scale_count:
            assert info.rc_s == 0
            assert np.array_equal(device_bytes(t.scales, 4 * t.scale_count),
                                  host_bytes(info.s, 4 * t.scale_count)), f"{info.name}: scales"
    ref.close()
    return m


def logits_of(runner, toks):
    out = []
    for t in toks:
        runner.forward(int(t))
        out.append(runner.logits())
    runner.close()
    return np.stack(out)


def assert_logits(got, want, tol=TOL):
    for t in range(want.shape[0]):
        err = np.abs(got[t] - want[t]).max()
        assert err <= tol * np.abs(want[t]).max(), f"token {t}: max err {err:.3e}"


@pytest.mark.parametrize("kv", [8, 2])
def test_f32_model_written_by_the_reference(dev, tmp_path, kv):
    """The engine's mock shape with random 2:4 masks and random norm
    weights, written by the reference's tb_tbm_create.  With kv < heads
    (GQA) the reference runner reads past k and v at position 0
    (ops.hpp:176), so only the device runners are compared there."""
    cfg, model = mock(seed=61, masks="rand", norms="rand", heads=8, kv=kv)
    path = tmp_path / "mock.tbm"
    F.write_ref(path, cfg, model)
    m = compare_with_reference(path)
    toks = np.random.default_rng(3).integers(0, cfg["vocab"], 24).astype(np.int32)
    got = logits_of(m.runner(), toks)
    assert np.array_equal(got, logits_of(T.Runner(cfg, model), toks))
    if kv == cfg["n_heads"]:
        assert_logits(got, F.ref_runner(path, toks, cfg["vocab"]))
    m.close()


def test_quantized_projections_stay_quantized(dev, tmp_path):
    """INT4 attention and INT8 MLP projections with their scales: bytes as
    the reference's views give them, and the runner over the loaded file
    equals the device runner over the same quantized weights."""
    cfg, model = mock(seed=62, masks="none", norms="rand", layers=2)
    entries = [("model.embed_tokens.weight", "f32", model["embed"])]
    qlayers, rlayers = [], []
    for l, ly in enumerate(model["layers"]):
        ql, rl = dict(ly), dict(ly)
        for n, comp in F.NAMES.items():
            w = ly[n][0]
            bits, gs = (4, 64) if n in ("q", "k", "v", "o") else (8, 128)
            data, scales = quantize(w, bits, gs)
            dt = T.INT4 if bits == 4 else T.INT8
            entries.append((f"model.layers.{l}.{comp}.weight", f"int{bits}",
                            (data, scales, w.shape[0], w.shape[1], gs)))
            ql[n] = (T.QuantWeight(data, dt, w.shape[0], w.shape[1], scales, gs), None)
            rl[n] = (O.dequant(dt, data, scales, gs, w.size).reshape(w.shape), None)
        entries += [(f"model.layers.{l}.input_layernorm.weight", "f32", ly["in_norm"]),
                    (f"model.layers.{l}.post_attention_layernorm.weight", "f32", ly["post_norm"])]
        qlayers.append(ql)
        rlayers.append(rl)
    entries += [("model.norm.weight", "f32", model["final_norm"]),
                ("lm_head.weight", "f32", model["lm_head"])]
    path = tmp_path / "quant.tbm"
    F.write_quant(path, cfg, entries)
    m = compare_with_reference(path)
    toks = np.random.default_rng(4).integers(0, cfg["vocab"], 16).astype(np.int32)
    got = logits_of(m.runner(), toks)
    assert np.array_equal(got, logits_of(T.Runner(cfg, dict(model, layers=qlayers)), toks))
    assert_logits(got, O.runner_run(cfg, dict(model, layers=rlayers), toks))
    m.close()


def test_bad_magic_and_truncation(dev, tmp_path):
    """A tensor whose header is not a .tb header loads without bytes and
    reports TB_ERR_BAD_MAGIC, as the reference's view does; a tensor whose
    bytes run past the end of the file fails the load (TB_ERR_TRUNCATED),
    where the reference would read out of bounds."""
    cfg, model = mock(seed=63, masks="none", layers=1)
    entries = [(n, "f32", w) for n, w, _ in F.tensors_of(cfg, model, dense_masks=False)]
    bad = "model.layers.0.mlp.up_proj.weight"
    path = tmp_path / "bad.tbm"
    F.write_quant(path, cfg, entries, bad_magic={bad})
    m = compare_with_reference(path)
    code, _ = m.tensor(m.find(bad))
    assert code == 5  # TB_ERR_BAD_MAGIC
    m.close()
    raw = bytearray(path.read_bytes())
    n = int.from_bytes(raw[-4:], "little")
    import json
    idx = json.loads(raw[-4 - n:-4])
    idx["tensors"][1]["num_weights"] = 10 ** 9  # runs past the end of the file
    js = json.dumps(idx).encode()
    path2 = tmp_path / "trunc.tbm"
    path2.write_bytes(bytes(raw[:-4 - n]) + js + len(js).to_bytes(4, "little"))
    with pytest.raises(T.TbError) as e:
        T.TbmModel(path2)
    assert e.value.code == 11  # TB_ERR_TRUNCATED
