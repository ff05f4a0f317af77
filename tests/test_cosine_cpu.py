"""The cosine-similarity case on the CPU: its oracle against the reference's own outputs (golden
fixtures), its Case surface against the reference's defaults and input stream, and the C ABI
symbols of include/cos_sm100.h."""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from golden_util import cos_names, load
from oracle import cos_oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "nl2cuda-kernel-agent_b200")


@pytest.mark.parametrize("name", cos_names())
def test_oracle_matches_reference_fixture(name):
    z = load(name)
    eps = float(z["eps"])
    S = cos_oracle.forward(z["A"], z["B"], eps)
    dA, dB = cos_oracle.backward(z["A"], z["B"], z["dS"], eps)
    # fp64 oracle vs the reference's fp32 evaluation: fp32 rounding of sums of D terms (S) and
    # of N or M terms (gradients).
    for got, ref in ((S, z["S"]), (dA, z["dA"]), (dB, z["dB"])):
        assert got.shape == ref.shape
        if ref.size:
            assert np.max(np.abs(got - ref)) <= 2e-5 + 2e-5 * np.max(np.abs(ref))


def test_fixture_set_covers_the_edge_cases():
    got = set(cos_names())
    for want in ("cos_empty_n0_m5_d3", "cos_single_n1_m1_d1", "cos_aligned_n9_m11_d16",
                 "cos_wide_n24_m20_d130", "cos_ragged_n45_m33_d40"):
        assert want in got


def test_oracle_properties():
    r = np.random.default_rng(5)
    A = r.standard_normal((30, 12))
    B = r.standard_normal((20, 12))
    S = cos_oracle.forward(A, B, 1e-8)
    assert np.abs(S).max() <= 1 + 1e-12
    # Scale invariance of S: the gradient is orthogonal to each row (up to eps / |a|).
    dA, dB = cos_oracle.backward(A, B, r.standard_normal((30, 20)), 1e-8)
    assert np.abs((dA * A).sum(1)).max() < 1e-6
    assert np.abs((dB * B).sum(1)).max() < 1e-6
    # Against central differences of the forward.
    dS = r.standard_normal((30, 20))
    h = 1e-6
    for (i, d) in [(0, 0), (7, 5), (29, 11)]:
        Ap, Am = A.copy(), A.copy()
        Ap[i, d] += h
        Am[i, d] -= h
        num = ((cos_oracle.forward(Ap, B, 1e-8) - cos_oracle.forward(Am, B, 1e-8)) * dS).sum()
        assert abs(num / (2 * h) - cos_oracle.backward(A, B, dS, 1e-8)[0][i, d]) < 1e-6


def test_case_fields_match_reference_defaults():
    from cases.cosine_sim import CASE, config
    assert CASE.name == "cosine_sim"
    assert CASE.params == {"eps": 1e-8}
    assert CASE.grad_inputs == ["A", "B"]
    assert CASE.dtype == "float32"
    if not any(k in os.environ for k in ("COS_N", "COS_M", "COS_D")):
        assert (config.N, config.M, config.D) == (2048, 2048, 64)


@pytest.mark.parametrize("seed,n,m", [(0, 96, 80), (2, 64, 64)])
def test_make_inputs_reproduces_reference_stream(seed, n, m):
    # A child process reads COS_N / COS_M at import, as the reference's config does.
    code = (
        "import sys, numpy as np, torch; sys.path.insert(0, %r);"
        "from cases.cosine_sim.reference import make_inputs;"
        "d = make_inputs(%d, torch.float32, 'cpu');"
        "np.savez(sys.argv[1], A=d['A'].numpy(), B=d['B'].numpy())" % (PKG, seed))
    out = os.path.join(ROOT, "_work", f"cos_mi_{seed}_{n}_{m}.npz")
    os.makedirs(os.path.dirname(out), exist_ok=True)
    env = dict(os.environ, COS_N=str(n), COS_M=str(m), COS_D="64")
    subprocess.run([sys.executable, "-c", code, out], check=True, env=env)
    got = np.load(out)
    z = load(f"cos_makeinputs_seed{seed}_n{n}_m{m}")
    np.testing.assert_array_equal(got["A"], z["A"])
    np.testing.assert_array_equal(got["B"], z["B"])
    os.remove(out)


@pytest.mark.parametrize("name", ["cos_makeinputs_seed0_n96_m80", "cos_aligned_n9_m11_d16",
                                  "cos_empty_n0_m5_d3"])
def test_reference_forward_and_autograd_match_fixture(name):
    from cases.cosine_sim.reference import reference_forward
    z = load(name)
    A = torch.from_numpy(z["A"]).requires_grad_(True)
    B = torch.from_numpy(z["B"]).requires_grad_(True)
    S = reference_forward({"A": A, "B": B}, {"eps": float(z["eps"])})
    S.backward(torch.from_numpy(z["dS"]))
    np.testing.assert_allclose(S.detach().numpy(), z["S"], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(A.grad.numpy(), z["dA"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(B.grad.numpy(), z["dB"], rtol=1e-5, atol=1e-6)


def test_native_refuses_cpu_tensors():
    from cases.cosine_sim import op
    A, B = torch.randn(4, 8), torch.randn(5, 8)
    with pytest.raises(RuntimeError):
        op.candidate({"A": A, "B": B}, {"eps": 1e-8})
