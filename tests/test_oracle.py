"""The CPU oracle against the reference's own outputs (golden fixtures) and against its numpy
restatement."""
import numpy as np
import pytest

from golden_util import load, names
from oracle import oracle


@pytest.mark.parametrize("name", names())
def test_oracle_matches_reference_fixture(name):
    z = load(name)
    g = float(z["gamma"])
    K = oracle.forward(z["X"], z["Y"], g)
    dX, dY = oracle.backward(z["X"], z["Y"], z["G"], g)
    # The fixture is the reference's fp32 evaluation; the oracle is fp64.  They agree to
    # fp32 rounding of sums of D and of N or M terms.
    for got, ref in ((K, z["K"]), (dX, z["dX"]), (dY, z["dY"])):
        assert got.shape == ref.shape
        if ref.size:
            assert np.max(np.abs(got - ref)) <= 2e-5 + 2e-5 * np.max(np.abs(ref))


def test_oracle_c_matches_numpy_restatement():
    r = np.random.default_rng(7)
    for (N, M, D, g) in [(5, 7, 3, 0.3), (31, 17, 64, 1 / 64), (1, 40, 130, 0.01)]:
        X = r.standard_normal((N, D)).astype(np.float32)
        Y = r.standard_normal((M, D)).astype(np.float32)
        G = r.standard_normal((N, M)).astype(np.float32)
        np.testing.assert_allclose(oracle.forward(X, Y, g), oracle.numpy_forward(X, Y, g),
                                   rtol=1e-12, atol=1e-14)
        dX, dY = oracle.backward(X, Y, G, g)
        rx, ry = oracle.numpy_backward(X, Y, G, g)
        np.testing.assert_allclose(dX, rx, rtol=1e-10, atol=1e-12)
        np.testing.assert_allclose(dY, ry, rtol=1e-10, atol=1e-12)


def test_oracle_subsets_match_full():
    r = np.random.default_rng(3)
    X = r.standard_normal((50, 9)).astype(np.float32)
    Y = r.standard_normal((40, 9)).astype(np.float32)
    G = r.standard_normal((50, 40)).astype(np.float32)
    K = oracle.forward(X, Y, 0.1)
    dX, dY = oracle.backward(X, Y, G, 0.1)
    rows = np.array([0, 17, 49, 3])
    cols = np.array([39, 0, 5])
    np.testing.assert_array_equal(oracle.forward_rows(X, Y, 0.1, rows), K[rows])
    np.testing.assert_array_equal(oracle.dx_rows(X, Y, G, 0.1, rows), dX[rows])
    np.testing.assert_array_equal(oracle.dy_cols(X, Y, G, 0.1, cols), dY[cols])


def test_translation_invariance_of_oracle():
    # K depends on x - y only, so sum_i dX_i + sum_j dY_j = 0: the size-independent property
    # the full-size GPU tests rely on.
    r = np.random.default_rng(11)
    X = r.standard_normal((20, 6)).astype(np.float32)
    Y = r.standard_normal((30, 6)).astype(np.float32)
    G = r.standard_normal((20, 30)).astype(np.float32)
    dX, dY = oracle.backward(X, Y, G, 0.2)
    assert np.abs(dX.sum(0) + dY.sum(0)).max() < 1e-12


def test_gate_helpers():
    assert oracle.allclose_gate([1.0, 2.0], [1.0005, 2.0], 1e-3, 1e-3)
    assert not oracle.allclose_gate([1.0], [1.1], 1e-3, 1e-3)
    a, r = oracle.max_errors([1.0, 2.0], [1.0, 2.5])
    assert a == pytest.approx(0.5) and r == pytest.approx(0.2)
