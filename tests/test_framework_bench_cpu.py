"""Host logic of the speed gate (framework/bench.py) and the protocol values, on the CPU: the
geometric mean, the coefficient-of-variation retry rule, and the refusal to time without CUDA."""
import pytest

from framework import bench
from framework.protocol import PROTOCOL


def test_protocol_keeps_the_reference_values():
    p = PROTOCOL
    assert (p.atol, p.rtol, p.seeds) == (1e-2, 1e-2, (0, 1, 2, 3, 4))
    assert (p.warmup, p.iters, p.repeats) == (10, 100, 3)
    assert (p.cv_threshold, p.max_retries, p.speedup_target) == (0.05, 4, 1.05)
    assert p.parity_tol == 1e-3


def test_geomean():
    assert bench._geomean([1.0, 4.0]) == pytest.approx(2.0)
    assert bench._geomean([3.0, 3.0, 3.0]) == pytest.approx(3.0)


def test_stable_retries_until_the_cv_is_in_bounds():
    rounds = iter([[1.0, 2.0, 3.0], [1.0, 1.5, 2.0], [1.0, 1.01, 0.99], [5.0, 5.0, 5.0]])
    s = bench._stable("forward", lambda: next(rounds))
    assert s["ok"] and s["attempts"] == 3
    assert s["geomeans_ms"] == [1.0, 1.01, 0.99]


def test_stable_keeps_the_lowest_cv_attempt_when_none_is_in_bounds():
    noisy = [[1.0, 3.0, 5.0], [1.0, 2.0, 3.0], [1.0, 4.0, 7.0], [1.0, 5.0, 9.0], [1.0, 3.0, 5.0]]
    rounds = iter(noisy)
    s = bench._stable("backward", lambda: next(rounds))
    assert not s["ok"]
    assert s["attempts"] == 2  # [1, 2, 3] has the lowest CV of the five
    assert s["geomeans_ms"] == [1.0, 2.0, 3.0]


def test_compare_refuses_to_time_without_cuda():
    from cases.cosine_sim import CASE
    from cases.cosine_sim.op import candidate
    with pytest.raises(RuntimeError, match="CUDA"):
        bench.compare(CASE, candidate, device="cpu")
