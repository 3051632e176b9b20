"""GPU parity: every sm_100a kernel, called through the C ABI of
libtb_b200.so, against the CPU oracle on the same seeded inputs.

Criteria (tests/parity.py): bit-exact for gather/argmax/adds/RoPE-at-table
positions; f32 row-wise relative error <= 1e-5; bf16 within 1 ulp of the
oracle's bf16 mode.  Shapes: the reference configs (mock, Llama-7B prefill,
decode, Llama-70B rows) plus the edges the kernels branch on (one row, odd
widths, unaligned pointers, rows too wide for registers, empty inputs, NaN,
+-inf, out-of-range ids).
"""
import ctypes as C

import numpy as np
import pytest

import tb_b200 as T
import workloads as W
from oracle import oracle as O
from parity import assert_bf16, assert_bitexact, assert_f32, blocks, from_np, to_np

pytestmark = pytest.mark.gpu

bf = O.f32_to_bf16


@pytest.fixture(scope="module")
def dev(cuda):
    import torch
    torch.cuda.set_device(cuda)
    return cuda


def gpu(a, dev):
    return from_np(a, dev)


def sync():
    import torch
    torch.cuda.synchronize()


def close(g, c, what, is_bf16):
    if is_bf16:
        return assert_bf16(g, c, what)
    return assert_f32(g, c, what)


# ------------------------------------------------------------------ KATs
def test_reference_kats_on_gpu(dev):
    # tests/test_norm.c:23-57 and tests/test_softmax.c:33-68, on the device.
    import torch
    x = torch.tensor([[1, 2, 3, 4]], dtype=torch.float32, device=dev)
    y = T.rms_norm(x, torch.ones(4, device=dev), 1e-6)
    np.testing.assert_allclose(to_np(y)[0], [1, 2, 3, 4] / np.sqrt(7.5 + 1e-6), atol=1e-4)
    y = T.rms_norm(torch.full((1, 4), 2.0, device=dev),
                   torch.tensor([0.5, 1, 1.5, 2], device=dev), 0.0)
    np.testing.assert_allclose(to_np(y)[0], [0.5, 1, 1.5, 2], atol=1e-4)
    s = to_np(T.softmax(torch.tensor([[1.0, 2, 3]], device=dev)))[0]
    assert abs(s.sum() - 1) <= 1e-4 and s[2] > s[1] > s[0]
    np.testing.assert_allclose(to_np(T.softmax(torch.full((1, 4), 5.0, device=dev))), 0.25,
                               atol=1e-4)
    s = to_np(T.softmax(torch.tensor([[1.0, 2, 3]], device=dev),
                        torch.tensor([[0.0, 0, -100]], device=dev)))[0]
    assert abs(s[2]) <= 1e-3 and s[1] > s[0]


# --------------------------------------------------------- residual+norm
NORM_SHAPES = [(64, 256), (4096, 4096), (256, 4096), (33, 100), (5, 16384), (7, 8192),
               (3, 40000), (1, 1), (2, 65536 + 8)]


@pytest.mark.parametrize("rows,cols", NORM_SHAPES)
@pytest.mark.parametrize("is_bf16", [False, True])
def test_residual_rms_norm(dev, rows, cols, is_bf16):
    cfg = W.CONFIGS["7b"]
    x = W.normal(cfg, 0, (rows, cols))
    r = W.normal(cfg, 1, (rows, cols))
    w = W.normal(cfg, 2, (cols,), std=0.1, mean=1.0)
    if is_bf16:
        x, r, w = bf(x), bf(r), bf(w)
    h_ref, y_ref = O.residual_rms_norm(x, r, w, 1e-5, threads=8)
    gx, gr, gw = gpu(x, dev), gpu(r, dev), gpu(w, dev)
    import torch
    gh = torch.empty_like(gx)
    _, gy = T.residual_rms_norm(gx, gr, gw, 1e-5, h_out=gh)
    sync()
    assert_bitexact(to_np(gh), h_ref, "h = x + residual")
    close(to_np(gy), y_ref, f"y {rows}x{cols}", is_bf16)


@pytest.mark.parametrize("is_bf16", [False, True])
def test_rms_norm_without_weight_or_residual(dev, is_bf16):
    rng = np.random.default_rng(4)
    x = rng.standard_normal((19, 1536), dtype=np.float32)
    if is_bf16:
        x = bf(x)
    y_ref = O.rms_norm(x, None, 1e-6)
    gy = T.rms_norm(gpu(x, dev), None, 1e-6)
    sync()
    close(to_np(gy), y_ref, "rms_norm, no weight", is_bf16)


def test_residual_rms_norm_in_place_and_unaligned(dev):
    import torch
    rng = np.random.default_rng(8)
    rows, cols = 40, 2048
    x = rng.standard_normal((rows, cols), dtype=np.float32)
    r = rng.standard_normal((rows, cols), dtype=np.float32)
    w = (1 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    h_ref, y_ref = O.residual_rms_norm(x, r, w, 1e-5)
    # in place: h overwrites the residual stream, y overwrites x
    gx, gr = gpu(x, dev), gpu(r, dev)
    T.lib().tb_b200_residual_rms_norm(T.F32, rows, cols, T.ptr(gx), T.ptr(gr),
                                      T.ptr(gpu(w, dev)), T.ptr(gr), T.ptr(gx), 1e-5, None)
    sync()
    assert_bitexact(to_np(gr), h_ref, "in-place h")
    assert_f32(to_np(gx), y_ref, "in-place y")
    # unaligned (4-byte offset) buffers take the scalar path
    bx = torch.zeros(rows * cols + 1, device=dev)
    br = torch.zeros(rows * cols + 1, device=dev)
    bx[1:] = gpu(x, dev).reshape(-1)
    br[1:] = gpu(r, dev).reshape(-1)
    out = torch.zeros(rows * cols + 1, device=dev)
    rc = T.lib().tb_b200_residual_rms_norm(T.F32, rows, cols, C.c_void_p(bx.data_ptr() + 4),
                                           C.c_void_p(br.data_ptr() + 4), T.ptr(gpu(w, dev)),
                                           None, C.c_void_p(out.data_ptr() + 4), 1e-5, None)
    assert rc == 0
    sync()
    assert_f32(to_np(out)[1:].reshape(rows, cols), y_ref, "unaligned y")


def test_norm_argument_errors(dev):
    L = T.lib()
    assert L.tb_b200_residual_rms_norm(T.F32, -1, 4, None, None, None, None, None, 1e-5, None) == 9
    assert L.tb_b200_residual_rms_norm(T.F32, 0, 4, None, None, None, None, None, 1e-5, None) == 0
    assert L.tb_b200_residual_rms_norm(T.I32, 2, 4, C.c_void_p(16), None, None, None,
                                       C.c_void_p(16), 1e-5, None) == 10
    assert L.tb_b200_rms_norm(T.F32, 2, 4, None, None, None, 1e-5, None) == 8


# ------------------------------------------------------------ elementwise
EW_N = [64 * 1024, 4096 * 11008, 1000003, 7, 1]


@pytest.mark.parametrize("n", EW_N)
@pytest.mark.parametrize("is_bf16", [False, True])
def test_elementwise(dev, n, is_bf16):
    cfg = W.CONFIGS["7b"]
    g = W.normal(cfg, 5, (1, n)) * np.float32(3)
    u = W.normal(cfg, 6, (1, n))
    if is_bf16:
        g, u = bf(g), bf(u)
    gg, gu = gpu(g, dev), gpu(u, dev)
    outs = {"silu": T.silu(gg), "gelu": T.gelu(gg), "swiglu": T.swiglu(gg, gu),
            "add": T.residual_add(gg, gu)}
    sync()
    for name, ref in [("silu", O.silu(g, threads=8)), ("gelu", O.gelu(g, threads=8)),
                      ("swiglu", O.swiglu(g, u, threads=8))]:
        close(blocks(to_np(outs[name])), blocks(ref), f"{name} n={n}", is_bf16)
    assert_bitexact(to_np(outs["add"]), O.residual_add(g, u), f"add n={n}")


def test_elementwise_unaligned_and_special_values(dev):
    import torch
    vals = np.array([0.0, -0.0, 1e-30, -1e-30, 88.0, -88.0, 100.0, -100.0, np.inf, -np.inf,
                     np.nan, 3.5, -3.5, 1e6, -1e6, 0.5], np.float32)
    buf = torch.zeros(vals.size + 1, device=dev)
    buf[1:] = gpu(vals, dev)
    src = C.c_void_p(buf.data_ptr() + 4)
    out = torch.zeros(vals.size + 1, device=dev)
    dst = C.c_void_p(out.data_ptr() + 4)
    for name, fn, ref in [("silu", T.lib().tb_b200_silu, O.silu),
                          ("gelu", T.lib().tb_b200_gelu, O.gelu)]:
        assert fn(T.F32, vals.size, src, dst, None) == 0
        sync()
        got = to_np(out)[1:]
        want = ref(vals[None])[0]
        assert (np.isnan(got) == np.isnan(want)).all(), name
        ok = ~np.isnan(want)
        # absolute floor: GELU's 1 + tanhf cancels for x < -3 (see parity.py)
        np.testing.assert_allclose(got[ok], want[ok], rtol=1e-5, atol=1e-5, err_msg=name)


# -------------------------------------------------------------------- RoPE
ROPE_CASES = [
    ("mock", 64, 4, 4, 64, 1e4, "arange"),
    ("7b", 4096, 32, 32, 128, 1e4, "arange"),
    ("decode", 256, 32, 32, 128, 1e4, "uniform4096"),
    ("70b", 512, 64, 8, 128, 5e5, "uniform16384"),
]


def _positions(kind, rows, seed):
    if kind == "arange":
        return np.arange(rows, dtype=np.int32)
    hi = int(kind.replace("uniform", ""))
    return np.random.default_rng(seed).integers(0, hi, rows).astype(np.int32)


@pytest.mark.parametrize("name,rows,hq,hkv,d,theta,pos_kind", ROPE_CASES)
@pytest.mark.parametrize("is_bf16", [False, True])
def test_rope_rows_table_is_bit_exact(dev, name, rows, hq, hkv, d, theta, pos_kind, is_bf16):
    rng = np.random.default_rng(rows + hq)
    q = rng.standard_normal((rows, hq, d), dtype=np.float32)
    k = rng.standard_normal((rows, hkv, d), dtype=np.float32)
    if is_bf16:
        q, k = bf(q), bf(k)
    pos = _positions(pos_kind, rows, rows)
    q_ref, k_ref = O.rope(q, k, pos, theta, threads=8)
    table = T.rope_table(theta, d, int(pos.max()) + 1)
    gq, gk = gpu(q, dev), gpu(k, dev)
    T.rope_rows(gq, gk, gpu(pos, dev), theta, table)
    sync()
    # identical cos/sin and identical rounding: bit-exact in f32; the bf16
    # result is the rounding of the bit-exact f32 one
    assert_bitexact(to_np(gq), q_ref, f"{name} q")
    assert_bitexact(to_np(gk), k_ref, f"{name} k")


@pytest.mark.parametrize("is_bf16", [False, True])
def test_rope_rows_outside_table_uses_device_sincos(dev, is_bf16):
    rng = np.random.default_rng(21)
    rows, hq, hkv, d, theta = 300, 8, 2, 128, 5e5
    q = rng.standard_normal((rows, hq, d), dtype=np.float32)
    k = rng.standard_normal((rows, hkv, d), dtype=np.float32)
    if is_bf16:
        q, k = bf(q), bf(k)
    pos = rng.integers(-50, 20000, rows).astype(np.int32)
    q_ref, k_ref = O.rope(q, k, pos, theta)
    table = T.rope_table(theta, d, 1000)  # most positions fall outside
    gq, gk = gpu(q, dev), gpu(k, dev)
    T.rope_rows(gq, gk, gpu(pos, dev), theta, table)
    sync()
    close(to_np(gq), q_ref, "q outside table", is_bf16)
    close(to_np(gk), k_ref, "k outside table", is_bf16)
    # no table at all
    gq, gk = gpu(q, dev), gpu(k, dev)
    T.rope_rows(gq, gk, gpu(pos, dev), theta, None)
    sync()
    close(to_np(gq), q_ref, "q without table", is_bf16)


def test_rope_single_position_and_odd_head_dim(dev):
    rng = np.random.default_rng(2)
    for hq, hkv, d, pos in [(32, 8, 128, 4095), (4, 4, 64, 0), (3, 1, 6, 77), (2, 2, 10, 9)]:
        q = rng.standard_normal((1, hq, d), dtype=np.float32)
        k = rng.standard_normal((1, hkv, d), dtype=np.float32)
        q_ref, k_ref = O.rope(q, k, np.array([pos], np.int32), 1e4)
        gq, gk = gpu(q[0], dev), gpu(k[0], dev)
        T.rope(gq, gk, pos, 1e4)
        sync()
        assert_bitexact(to_np(gq), q_ref[0], f"rope d={d} q")
        assert_bitexact(to_np(gk), k_ref[0], f"rope d={d} k")


# ----------------------------------------------------------------- softmax
# By default f32 rows of up to 32768 columns (a multiple of 4, no mask,
# aligned) take the shared-memory-staged kernel and the rest the tiled one;
# with TB_B200_SOFTMAX=cluster, rows of 1024 to 131072 such columns take the
# cluster kernel (C = ceil(tiles / 64) CTAs per row, 256-term tiles).
# "pipeline" gives every CTA many rows (cluster: C = 1); "staged_max" the
# widest staged row (C = 2) and "past_staged" the first width beyond it (C =
# 3, a last tile of 4 terms); "c5" 5 CTAs of 64 tiles; "c3_ragged" a last
# tile of 4 terms; "cluster_max" the cluster kernel's widest row (8 CTAs of
# 64 tiles); "c8_spiky" many binade crossings; bf16 takes the tiled kernel.
SOFTMAX_CASES = [("mock", 64, 100, 2.0), ("7b", 256, 32000, 3.0), ("70b", 16, 128256, 3.0),
                 ("odd", 9, 1001, 3.0), ("one", 3, 1, 1.0), ("wide_std", 8, 5000, 20.0),
                 ("pipeline", 600, 4096, 3.0), ("staged_max", 300, 32768, 3.0),
                 ("past_staged", 5, 32772, 3.0), ("spiky", 40, 32000, 12.0),
                 ("c5", 33, 81920, 3.0), ("c3_ragged", 17, 40964, 3.0),
                 ("cluster_max", 20, 131072, 3.0), ("c8_spiky", 40, 128256, 12.0),
                 ("min_cluster", 50, 1024, 3.0)]


@pytest.mark.parametrize("name,rows,cols,std", SOFTMAX_CASES)
@pytest.mark.parametrize("is_bf16", [False, True])
def test_softmax(dev, name, rows, cols, std, is_bf16):
    x = np.random.default_rng(cols).standard_normal((rows, cols), dtype=np.float32) * \
        np.float32(std)
    if is_bf16:
        x = bf(x)
    y_ref = O.softmax(x, None, threads=8)
    gy = T.softmax(gpu(x, dev))
    sync()
    close(to_np(gy), y_ref, f"softmax {name}", is_bf16)


def test_softmax_sum_is_the_sequential_sum(dev):
    """At 128K terms a tree sum misses the reference's sequential f32 sum by
    ~1e-4; the kernel must reproduce it.  Checked through 1/sum: with
    expf within 2 ulp, y*sum recovers the row's own exponentials."""
    rng = np.random.default_rng(77)
    x = rng.standard_normal((4, 128256), dtype=np.float32) * np.float32(3)
    y_ref = O.softmax(x)
    gy = to_np(T.softmax(gpu(x, dev)))
    sync()
    worst, _ = assert_f32(gy, y_ref, "softmax 128K")
    assert worst < 2e-6, f"softmax 128K row error {worst:.2e}: not the sequential sum"


@pytest.fixture
def cluster_softmax(monkeypatch):
    """Route f32 softmax to the cluster kernel (k_softmax_cluster.cu)."""
    monkeypatch.setenv("TB_B200_SOFTMAX", "cluster")


@pytest.mark.parametrize("name,rows,cols,std", [c for c in SOFTMAX_CASES if c[2] >= 1024])
def test_cluster_softmax(dev, cluster_softmax, name, rows, cols, std):
    """The cluster kernel on every f32 case wide enough for it."""
    x = np.random.default_rng(cols).standard_normal((rows, cols), dtype=np.float32) * \
        np.float32(std)
    y_ref = O.softmax(x, None, threads=8)
    gy = T.softmax(gpu(x, dev))
    sync()
    worst, _ = assert_f32(to_np(gy), y_ref, f"cluster softmax {name}")
    assert worst < 2e-6, f"cluster softmax {name}: row error {worst:.2e}"
    assert T.check_status() == (0, 0)


@pytest.mark.parametrize("std", [3.0, 12.0])
@pytest.mark.parametrize("cluster", [False, True])
def test_cluster_softmax_sum_over_many_rows(dev, monkeypatch, std, cluster):
    """400 rows of 128256 terms, through the default kernel and through the
    cluster kernel, where every cluster takes many rows, so its segment
    buffers, exchange slots and scanner keys all wrap around.  Each row must
    still be the sequential sum (row error < 2e-6)."""
    if cluster:
        monkeypatch.setenv("TB_B200_SOFTMAX", "cluster")
    rng = np.random.default_rng(79 + int(std))
    x = rng.standard_normal((400, 128256), dtype=np.float32) * np.float32(std)
    y_ref = O.softmax(x, threads=8)
    gy = to_np(T.softmax(gpu(x, dev)))
    sync()
    worst, _ = assert_f32(gy, y_ref, f"cluster softmax std {std}")
    assert worst < 2e-6, f"cluster softmax std {std}: row error {worst:.2e}"
    assert T.check_status() == (0, 0)


@pytest.mark.parametrize("cluster", [False, True])
def test_softmax_in_place_and_nan_in_wide_rows(dev, monkeypatch, cluster):
    """y may alias x; a NaN term makes its row NaN, other rows unaffected."""
    if cluster:
        monkeypatch.setenv("TB_B200_SOFTMAX", "cluster")
    rng = np.random.default_rng(5)
    x = rng.standard_normal((300, 32000), dtype=np.float32) * np.float32(3)
    x[7, 20000] = np.float32("nan")
    x[8, :] = -np.inf
    x[9, 31999] = np.inf
    x[10, 5] = np.float32(3e38)  # a row max beyond the fused exponent's range
    x[11, :] = np.float32(1e30)
    y_ref = O.softmax(x)
    g = gpu(x, dev)
    T.softmax(g, y=g)
    sync()
    gy = to_np(g)
    assert (np.isnan(gy) == np.isnan(y_ref)).all()
    keep = ~np.isnan(y_ref).any(axis=1)
    assert_f32(gy[keep], y_ref[keep], "softmax in place")
    # NaN rows are left unnormalised, as the reference leaves them
    assert_f32(gy[7][~np.isnan(y_ref[7])][None], y_ref[7][~np.isnan(y_ref[7])][None],
               "softmax NaN row")
    assert T.check_status() == (0, 0)


@pytest.mark.parametrize("masked", [False, True])
def test_softmax_special_rows_128k(dev, masked):
    """Rows of 128256 terms (the tiled kernel, in place) with the values
    that reach its slot tables' edge cases: NaN, all -inf, +inf, a max
    beyond the fused exponent's range, all equal (a sum of exact integers),
    a single spike, very spiky and near-uniform rows, tiny values; with a
    mask of -inf entries too.  Finite rows: the in-order sum (row error
    < 2e-6); NaN rows stay unnormalised, as in the reference."""
    rng = np.random.default_rng(81)
    n = 128256
    x = rng.standard_normal((12, n), dtype=np.float32) * np.float32(3)
    x[1, 100000] = np.float32("nan")
    x[2, :] = -np.inf
    x[3, 5] = np.inf
    x[4, 77] = np.float32(3e38)
    x[5, :] = np.float32(1e30)
    x[6, :] = 0.0
    x[7, :] = 0.0
    x[7, 50000] = 5.0
    x[8] *= np.float32(10)                          # std 30: a few terms dominate
    x[9] = rng.standard_normal(n).astype(np.float32) * np.float32(0.01)  # near-uniform
    x[10] = np.float32(-200) + rng.standard_normal(n).astype(np.float32)
    mask = None
    if masked:
        mask = rng.standard_normal((12, n), dtype=np.float32)
        mask[:, ::3] = -np.inf
        mask[11, :] = -np.inf                          # a fully masked row: NaN
    y_ref = O.softmax(x, mask, threads=8)
    g = gpu(x, dev)
    T.softmax(g, None if mask is None else gpu(mask, dev), y=g)
    sync()
    gy = to_np(g)
    assert (np.isnan(gy) == np.isnan(y_ref)).all()
    keep = ~np.isnan(y_ref).any(axis=1)
    worst, _ = assert_f32(gy[keep], y_ref[keep], "softmax 128K special rows")
    assert worst < 2e-6, f"softmax 128K special rows: row error {worst:.2e}"
    for r in np.nonzero(~keep)[0]:
        ok = ~np.isnan(y_ref[r])
        if ok.any():
            assert_f32(gy[r][ok][None], y_ref[r][ok][None], f"softmax 128K NaN row {r}")
    assert T.check_status() == (0, 0)


def test_staged_softmax_sum_is_the_sequential_sum(dev):
    """The shared-memory-staged path (f32, 32000 columns, many rows per CTA)
    must also return the in-order sum: row error < 2e-6, where a tree sum of
    the same terms misses by ~7e-5; std-12 rows cross many binades."""
    rng = np.random.default_rng(78)
    for std in (3.0, 12.0):
        x = rng.standard_normal((600, 32000), dtype=np.float32) * np.float32(std)
        y_ref = O.softmax(x, threads=8)
        gy = to_np(T.softmax(gpu(x, dev)))
        sync()
        worst, _ = assert_f32(gy, y_ref, f"staged softmax std {std}")
        assert worst < 2e-6, f"staged softmax std {std}: row error {worst:.2e}"


def test_softmax_with_mask_and_special_rows(dev):
    nan, inf = np.float32("nan"), np.float32("inf")
    x = np.array([[1, 2, 3, 4], [0, nan, 1, 2], [-inf, -inf, -inf, -inf], [inf, 1, 2, 3],
                  [5, 5, 5, 5], [-inf, 0, -inf, 1]], np.float32)
    mask = np.array([[0, 0, -100, 0]] * 6, np.float32)
    for m in (None, mask):
        y_ref = O.softmax(x, m)
        gy = to_np(T.softmax(gpu(x, dev), None if m is None else gpu(m, dev)))
        sync()
        assert (np.isnan(gy) == np.isnan(y_ref)).all()
        ok = ~np.isnan(y_ref)
        np.testing.assert_allclose(gy[ok], y_ref[ok], rtol=1e-6, atol=1e-7)


# ------------------------------------------------------------------ argmax
@pytest.mark.parametrize("rows,cols", [(64, 100), (256, 32000), (8, 128256), (5, 3001), (3, 1)])
@pytest.mark.parametrize("is_bf16", [False, True])
def test_argmax_bit_exact(dev, rows, cols, is_bf16):
    x = np.random.default_rng(rows * cols).standard_normal((rows, cols), dtype=np.float32)
    if is_bf16:
        x = bf(x)  # many ties: the first maximum must win
    got = to_np(T.argmax(gpu(x, dev)))
    sync()
    assert_bitexact(got, O.argmax(x), f"argmax {rows}x{cols}")


def test_argmax_edge_rows(dev):
    nan, inf = np.float32("nan"), np.float32("inf")
    rows = [[1, 3, 3, 2], [nan, 5, 7, 1], [1, nan, 0.5, 0], [-inf, -inf, -inf, -inf],
            [-inf, nan, -inf, nan], [-0.0, 0.0, -1, -2], [-5, -inf, inf, inf], [2, 2, 2, 2]]
    x = np.array(rows, np.float32)
    assert_bitexact(to_np(T.argmax(gpu(x, dev))), O.argmax(x), "argmax edges")
    wide = np.full((3, 70000), -inf, np.float32)
    wide[0, 0] = nan
    wide[1, 69999] = 1.0
    wide[1, 12345] = 1.0
    wide[2, 5] = -0.0
    wide[2, 40000] = 0.0
    assert_bitexact(to_np(T.argmax(gpu(wide, dev))), O.argmax(wide), "argmax wide edges")


# --------------------------------------------------------------- embedding
@pytest.mark.parametrize("cfg_name,n_tokens,vocab,hidden", [("mock", 64, 100, 256),
                                                            ("7b", 4096, 32000, 4096),
                                                            ("odd", 77, 1000, 33)])
@pytest.mark.parametrize("is_bf16", [False, True])
def test_embedding_bit_exact(dev, cfg_name, n_tokens, vocab, hidden, is_bf16):
    rng = np.random.default_rng(vocab)
    table = (rng.standard_normal((vocab, hidden), dtype=np.float32) * np.float32(0.02))
    if is_bf16:
        table = bf(table)
    ids = rng.integers(0, vocab, n_tokens).astype(np.int32)
    y = to_np(T.embedding(gpu(ids, dev), gpu(table, dev)))
    sync()
    assert_bitexact(y, O.embedding(ids, table), f"embedding {cfg_name}")
    rc, flags = T.check_status()
    assert rc == 0 and flags == 0


def test_embedding_out_of_range_ids_flag_and_zero(dev):
    import torch
    table = np.arange(40, dtype=np.float32).reshape(10, 4)
    ids = np.array([1, 10, -1, 3], np.int32)
    y = to_np(T.embedding(gpu(ids, dev), gpu(table, dev)))
    rc, flags = T.check_status()
    assert rc == 8 and flags == T.FLAG_TOKEN_RANGE
    assert (y[1] == 0).all() and (y[2] == 0).all()
    assert_bitexact(y[[0, 3]], table[[1, 3]], "valid rows")
    assert T.check_status() == (0, 0)  # cleared
    # host ids are checked on the host: nothing is queued
    out = torch.full((4, 4), 7.0, device=dev)
    rc = T.lib().tb_b200_embedding_host_ids(T.F32, 4, 4, 10, ids.ctypes.data,
                                            T.ptr(gpu(table, dev)), T.ptr(out), None)
    sync()
    assert rc == 8 and (to_np(out) == 7.0).all()


# ---------------------------------------------- registry with device tensors
def test_registry_routes_device_tensors_to_b200(dev):
    import torch
    L = T.lib()
    L.tb_backend_reset()
    assert L.tb_backend_b200_init() == 0
    try:
        rng = np.random.default_rng(13)
        x = rng.standard_normal((8, 512), dtype=np.float32)
        r = rng.standard_normal((8, 512), dtype=np.float32)
        w = (1 + 0.1 * rng.standard_normal(512)).astype(np.float32)
        gx, gr, gw = gpu(x, dev), gpu(r, dev), gpu(w, dev)
        gy, gh = torch.empty_like(gx), torch.empty_like(gx)
        tx, tr, tw, ty, th = map(T.tensor, (gx, gr, gw, gy, gh))
        assert L.tb_dispatch_residual_rms_norm(C.byref(ty), C.byref(th), C.byref(tx),
                                               C.byref(tr), C.byref(tw), C.c_float(1e-5)) == 0
        h_ref, y_ref = O.residual_rms_norm(x, r, w, 1e-5)
        sync()
        assert_bitexact(to_np(gh), h_ref, "dispatch h")
        assert_f32(to_np(gy), y_ref, "dispatch y")
        # rank-1 RMS_NORM is the engine's one-vector semantics
        v = gpu(x[0], dev)
        tv, tw1 = T.tensor(v), T.tensor(gw)
        out = torch.empty_like(v)
        to = T.tensor(out)
        assert L.tb_dispatch_rms_norm(C.byref(to), C.byref(tv), C.byref(tw1), C.c_float(1e-6)) == 0
        sync()
        assert_f32(to_np(out)[None], O.rms_norm(x[:1], w, 1e-6), "dispatch rank-1")
        # embedding with host ids, as TransformerRunner passes &token_id
        table = (rng.standard_normal((50, 64), dtype=np.float32) * np.float32(0.02))
        gt = gpu(table, dev)
        emb = torch.empty((3, 64), device=dev)
        ids = (C.c_int * 3)(4, 49, 0)
        te, tt = T.tensor(emb), T.tensor(gt)
        assert L.tb_dispatch_embedding(C.byref(te), ids, 3, C.byref(tt)) == 0
        sync()
        assert_bitexact(to_np(emb), table[[4, 49, 0]], "dispatch embedding")
        # ROPE (engine shape [heads, 1, d]) and ROPE_ROWS with host positions
        q = rng.standard_normal((1, 32, 128), dtype=np.float32)
        k = rng.standard_normal((1, 8, 128), dtype=np.float32)
        gq, gk = gpu(q[0].reshape(32, 1, 128), dev), gpu(k[0].reshape(8, 1, 128), dev)
        tq, tk = T.tensor(gq), T.tensor(gk)
        assert L.tb_dispatch_rope(C.byref(tq), C.byref(tk), 17, C.c_float(1e4), 128) == 0
        q_ref, k_ref = O.rope(q, k, np.array([17], np.int32), 1e4)
        sync()
        assert_bitexact(to_np(gq).reshape(1, 32, 128), q_ref, "dispatch rope q")
        assert_bitexact(to_np(gk).reshape(1, 8, 128), k_ref, "dispatch rope k")
        qs = rng.standard_normal((6, 32, 128), dtype=np.float32)
        ks = rng.standard_normal((6, 8, 128), dtype=np.float32)
        pos = np.array([0, 5, 4095, 100, 7, 3], np.int32)
        gq, gk = gpu(qs, dev), gpu(ks, dev)
        tq, tk = T.tensor(gq), T.tensor(gk)
        assert L.tb_dispatch_rope_rows(C.byref(tq), C.byref(tk), pos.ctypes.data, C.c_float(1e4),
                                       128, 4096) == 0
        q_ref, k_ref = O.rope(qs, ks, pos, 1e4)
        sync()
        assert_bitexact(to_np(gq), q_ref, "dispatch rope_rows q")
        assert_bitexact(to_np(gk), k_ref, "dispatch rope_rows k")
        # argmax into an I32 tensor
        lg = gpu(rng.standard_normal((5, 1000), dtype=np.float32), dev)
        am = torch.empty(5, dtype=torch.int32, device=dev)
        ta, tl = T.tensor(am), T.tensor(lg)
        assert L.tb_dispatch_argmax(C.byref(ta), C.byref(tl)) == 0
        sync()
        assert_bitexact(to_np(am), O.argmax(to_np(lg)), "dispatch argmax")
        # host tensors find no backend (only "b200" is registered)
        host = T.tensor(torch.zeros(4), device=T.DEVICE_CPU)
        assert L.tb_dispatch_silu(C.byref(host), C.byref(host)) == 14
    finally:
        L.tb_backend_reset()


# ------------------------------------------------------------- layer chain
def _chain_inputs(cfg, rows, is_bf16, dev):
    li = W.layer_inputs(cfg, rows=rows)
    cv = bf if is_bf16 else (lambda a: a)
    return {k: (gpu(cv(v), dev) if k != "pos" else gpu(v, dev)) for k, v in li.items()}, li


@pytest.mark.parametrize("cfg_name,rows,is_bf16", [("mock", 64, False), ("decode", 256, True),
                                                   ("7b", 512, False)])
def test_layer_chain_matches_separate_ops(dev, cfg_name, rows, is_bf16):
    import torch
    cfg = W.CONFIGS[cfg_name]
    g, raw = _chain_inputs(cfg, rows, is_bf16, dev)
    table = T.rope_table(cfg.theta, cfg.head_dim, 4096)
    # separate launches
    a = {k: v.clone() for k, v in g.items()}
    h1, y1, act1 = torch.empty_like(a["x"]), torch.empty_like(a["x"]), torch.empty_like(a["gate"])
    T.residual_rms_norm(a["x"], a["res"], a["gamma"], cfg.eps, h_out=h1, y=y1)
    T.rope_rows(a["q"], a["k"], a["pos"], cfg.theta, table)
    T.swiglu(a["gate"], a["up"], act1)
    # one fused launch
    b = {k: v.clone() for k, v in g.items()}
    h2, y2, act2 = torch.empty_like(b["x"]), torch.empty_like(b["x"]), torch.empty_like(b["gate"])
    T.layer_chain(T.make_chain(b["x"], b["res"], b["gamma"], h2, y2, cfg.eps, b["q"], b["k"],
                               b["pos"], cfg.theta, table, b["gate"], b["up"], act2))
    sync()
    for u, v, n in [(h1, h2, "h"), (y1, y2, "y"), (a["q"], b["q"], "q"), (a["k"], b["k"], "k"),
                    (act1, act2, "act")]:
        assert_bitexact(to_np(v), to_np(u), f"chain {n}")
    # and against the oracle
    cv = bf if is_bf16 else (lambda x: x)
    h_ref, y_ref = O.residual_rms_norm(cv(raw["x"]), cv(raw["res"]), cv(raw["gamma"]), cfg.eps,
                                       threads=8)
    assert_bitexact(to_np(h2), h_ref, "chain h vs oracle")
    close(to_np(y2), y_ref, "chain y vs oracle", is_bf16)
    close(to_np(act2), O.swiglu(cv(raw["gate"]), cv(raw["up"]), threads=8), "chain act",
          is_bf16)


def test_layer_chain_cuda_graph_over_32_layers(dev):
    """Decode step: 32 layers of the chain captured once, replayed as one
    graph launch; the replay gives the same bits as eager launches."""
    import torch
    cfg = W.CONFIGS["decode"]
    layers = []
    for l in range(4):  # distinct buffers for 4 layers, reused cyclically
        g, _ = _chain_inputs(W.Config(**{**cfg.__dict__, "seed": 3000 + 100 * l}), cfg.rows, True,
                             dev)
        g["h"] = torch.empty_like(g["x"])
        g["y"] = torch.empty_like(g["x"])
        g["act"] = torch.empty_like(g["gate"])
        layers.append(g)
    table = T.rope_table(cfg.theta, cfg.head_dim, 4096)
    snap = [{k: v.clone() for k, v in g.items()} for g in layers]
    chains = [T.make_chain(g["x"], g["res"], g["gamma"], g["h"], g["y"], cfg.eps, g["q"], g["k"],
                           g["pos"], cfg.theta, table, g["gate"], g["up"], g["act"])
              for g in layers]
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for l in range(32):
            T.layer_chain(chains[l % 4], stream=C.c_void_p(s.cuda_stream))
    s.synchronize()
    eager = [{k: v.clone() for k, v in g.items()} for g in layers]
    for g, sn in zip(layers, snap):
        for k in g:
            g[k].copy_(sn[k])
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        for l in range(32):
            T.layer_chain(chains[l % 4], stream=C.c_void_p(s.cuda_stream))
    graph.replay()
    torch.cuda.synchronize()
    for g, e in zip(layers, eager):
        for k in g:
            assert_bitexact(to_np(g[k]), to_np(e[k]), f"graph replay {k}")
