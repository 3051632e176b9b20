"""GPU parity of temperature sampling (tb_b200_sample_temperature) with the
reference's sample_temperature (src/main.cpp:91-111).

The reference draws from std::discrete_distribution with a std::mt19937
seeded from std::random_device; the device sampler takes the draw's uniform
value u per row instead.  Here u is the generate_canonical<double, 53> stream
of a seeded mt19937 (the oracle's restatement, pinned to libstdc++ in
tests/test_oracle.py), and every row's index must equal the oracle's.
"""
import numpy as np
import pytest

import tb_b200 as T
from oracle import oracle as O
from parity import from_np, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev(cuda):
    import torch
    torch.cuda.set_device(cuda)
    return cuda


def draw(dev, x, temperature, u):
    gx, gu = from_np(np.ascontiguousarray(x, np.float32), dev), from_np(np.asarray(u, np.float64), dev)
    out = T.sample_temperature(gx, temperature, gu)
    return to_np(out)


@pytest.mark.parametrize("temperature", [0.5, 0.8, 1.0, 1.5, 3.0])
def test_decode_batch_draws_match_reference(dev, temperature):
    """256 sequences x 32000 vocab, logits N(0, 3)."""
    rng = np.random.default_rng(21)
    x = (rng.standard_normal((256, 32000)) * 3).astype(np.float32)
    u = O.uniforms(1000 + int(temperature * 10), 256)
    assert np.array_equal(draw(dev, x, temperature, u), O.sample_temperature(x, temperature, u, 8))


def test_128k_vocab_draws_match_reference(dev):
    rng = np.random.default_rng(22)
    x = (rng.standard_normal((64, 128256)) * 3).astype(np.float32)
    u = O.uniforms(77, 64)
    assert np.array_equal(draw(dev, x, 1.0, u), O.sample_temperature(x, 1.0, u, 8))


def special_rows():
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((12, 1000)) * 3).astype(np.float32)
    x[1, 0] = np.nan                 # the reference's max stays NaN
    x[2, 500] = np.nan               # one NaN weight
    x[3, 7] = np.inf                 # max = +inf
    x[4, :] = -np.inf                # every weight NaN
    x[5, 100:] = -np.inf             # zero weights
    x[6, :] = 2.5                    # equal weights: cp_i = (i + 1) / n
    x[7, :] = np.float32(1e30)
    x[7, 3] = np.float32(-1e30)
    x[8, :] = 0.0
    x[8, 999] = 50.0                 # one weight dominates
    x[9, ::2] = -np.inf              # every other weight zero
    return x


@pytest.mark.parametrize("temperature", [1.0, 1e-4, 1e4, float("inf")])
def test_special_rows_match_reference(dev, temperature):
    x = special_rows()
    for seed in (1, 2, 3):
        u = O.uniforms(seed, x.shape[0])
        assert np.array_equal(draw(dev, x, temperature, u),
                              O.sample_temperature(x, temperature, u)), (temperature, seed)


def test_boundary_uniforms_take_the_in_order_path(dev):
    """Equal weights put cumulative boundaries at k / n: u exactly on one
    (and next to one) cannot be decided from the parallel prefix and must
    take the in-order path; u = 0 and u just below 1 are the ends."""
    n = 1024
    x = np.full((1, n), 1.25, np.float32)
    us = [0.0, 0.5, 0.25, 0.125, 0.75, 1.0 / 1024, 1023.0 / 1024, np.nextafter(1.0, 0.0),
          np.nextafter(0.5, 1.0), np.nextafter(0.5, 0.0), 1e-300]
    xs = np.repeat(x, len(us), axis=0)
    got = draw(dev, xs, 1.0, np.array(us))
    want = O.sample_temperature(xs, 1.0, np.array(us))
    assert np.array_equal(got, want), (got, want)
    assert got[0] == 0 and got[7] == n - 1


def test_argmax_and_single_column(dev):
    rng = np.random.default_rng(23)
    x = (rng.standard_normal((33, 5000)) * 3).astype(np.float32)
    u = O.uniforms(5, 33)
    for t in (0.0, -1.0):
        assert np.array_equal(draw(dev, x, t, u), O.sample_temperature(x, t, u))
    one = np.array([[3.0], [np.nan]], np.float32)
    assert np.array_equal(draw(dev, one, 1.0, np.array([0.3, 0.9])), [0, 0])
