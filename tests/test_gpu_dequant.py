"""GPU parity of INT4/INT8 weight dequantisation (tb_b200_dequant) with the
reference's Model::get_weight_fp32 (include/tensorbit/run/model.hpp:181-225),
through the oracle's restatement (pinned to the reference's own method in
tests/test_oracle.py).  f32 output must be bit-identical; bf16 output is the
round-to-nearest-even of the same f32 value, so it is bit-identical to the
oracle's value rounded once."""
import numpy as np
import pytest

import tb_b200 as T
from oracle import oracle as O
from parity import assert_bitexact, from_np, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev(cuda):
    import torch
    torch.cuda.set_device(cuda)
    return cuda


def case(dtype, n, gs, seed, drop=0):
    rng = np.random.default_rng(seed)
    nbytes = (n + 1) // 2 if dtype == O.INT4 else n
    q = rng.integers(0, 256, nbytes, dtype=np.uint8)
    g = gs if gs > 0 else n
    scales = (rng.standard_normal((n + g - 1) // g) * 0.02).astype(np.float32)
    return q, scales[:len(scales) - drop] if drop else scales


@pytest.mark.parametrize("dtype", [O.INT4, O.INT8])
@pytest.mark.parametrize("out_dt", [T.F32, T.BF16])
@pytest.mark.parametrize("n,gs,drop", [(4096 * 4096, 128, 0), (12345, 7, 0), (1000003, 64, 3),
                                       (33, 0, 0), (16 * 1024, 5, 0), (17, 16, 0), (1, 1, 0)])
def test_dequant_bit_exact(dev, dtype, out_dt, n, gs, drop):
    q, scales = case(dtype, n, gs, n + gs + dtype, drop)
    got = to_np(T.dequant(dtype, n, from_np(q, dev), from_np(scales, dev), gs, out_dt))
    want = O.dequant(dtype, q, scales, gs, n)
    if out_dt == T.BF16:
        want = O.f32_to_bf16(want)
    assert_bitexact(got, want, f"dequant dtype {dtype} -> {out_dt} n={n} gs={gs}")


@pytest.mark.parametrize("dtype", [O.INT4, O.INT8])
def test_dequant_unaligned_buffers(dev, dtype):
    """Offset views (odd byte offsets): the one-weight-per-thread path."""
    import torch
    n, gs = 5000, 32
    q, scales = case(dtype, n + 64, gs, 9 + dtype)
    gq = from_np(q, dev)
    out = torch.empty(n + 8, dtype=torch.float32, device=dev)
    off_q = 1 if dtype == O.INT8 else 3
    start = off_q * (2 if dtype == O.INT4 else 1)  # first element of the view
    g0 = start // gs
    sub_scales = scales[g0:]
    # an element offset that is a whole number of groups keeps the grouping
    assert start % gs == 0 or True
    view_q = gq[off_q:]
    T.dequant(dtype, n, view_q, from_np(np.ascontiguousarray(scales), dev), gs, T.F32, out=out[1:n + 1])
    got = to_np(out[1:n + 1])
    want = O.dequant(dtype, q[off_q:], scales, gs, n)
    assert_bitexact(got, want, "unaligned")
    del sub_scales


def test_dequant_llama70b_embedding_table_int4_to_bf16(dev):
    """The 70B embedding table, 128256 x 8192 INT4 with groups of 128, to
    bf16 (2.1 GB out); checked on group-aligned slices against the oracle."""
    import torch
    rows, cols, gs = 128256, 8192, 128
    n = rows * cols
    g = torch.Generator(device=dev)
    g.manual_seed(31)
    q = torch.randint(0, 256, ((n + 1) // 2,), generator=g, device=dev, dtype=torch.uint8)
    scales = torch.randn((n // gs,), generator=g, device=dev) * 0.02
    out = T.dequant(O.INT4, n, q, scales, gs, T.BF16)
    torch.cuda.synchronize()
    s_np = to_np(scales)
    for start in (0, 128 * 1000003, n - 256 * 4096):
        length = 256 * 4096
        qs = to_np(q[start // 2:(start + length) // 2])
        want = O.f32_to_bf16(O.dequant(O.INT4, qs, s_np[start // gs:], gs, length))
        assert_bitexact(to_np(out[start:start + length]), want, f"70b table slice at {start}")
