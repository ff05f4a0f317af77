"""The Case surface mirrors the reference's: config defaults, make_inputs stream, the
broadcast reference_forward and its autograd backward, pinned to the reference's own outputs."""
import importlib
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from golden_util import load

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "nl2cuda-kernel-agent_b200")


def test_case_fields_match_reference_defaults():
    from cases.rbf import CASE, config
    assert CASE.name == "rbf"
    assert CASE.params == {"gamma": 1.0 / 64.0}
    assert CASE.grad_inputs == ["X", "Y"]
    assert CASE.dtype == "float32"
    if "RBF_SIZE" not in os.environ and "RBF_N" not in os.environ:
        assert (config.N, config.M, config.D) == (2048, 2048, 64)


@pytest.mark.parametrize("seed,size", [(0, 128), (1, 64), (4, 64)])
def test_make_inputs_reproduces_reference_stream(seed, size, tmp_path):
    # Run in a child process so RBF_SIZE is read at import, as the reference's config does.
    code = (
        "import sys, numpy as np, torch; sys.path.insert(0, %r);"
        "from cases.rbf.reference import make_inputs;"
        "d = make_inputs(%d, torch.float32, 'cpu');"
        "np.savez(sys.argv[1], X=d['X'].numpy(), Y=d['Y'].numpy())" % (PKG, seed))
    out = str(tmp_path / f"mi_{seed}_{size}.npz")
    env = dict(os.environ, RBF_SIZE=str(size))
    subprocess.run([sys.executable, "-c", code, out], check=True, env=env)
    got = np.load(out)
    z = load(f"ref_makeinputs_seed{seed}_n{size}")
    np.testing.assert_array_equal(got["X"], z["X"])
    np.testing.assert_array_equal(got["Y"], z["Y"])


@pytest.mark.parametrize("name", ["ref_makeinputs_seed0_n128", "ragged_n37_m50_d5",
                                  "duplicates_n40_m49_d64", "empty_n0_m5_d3"])
def test_reference_forward_and_autograd_match_fixture(name):
    from cases.rbf.reference import reference_forward
    z = load(name)
    X = torch.from_numpy(z["X"]).requires_grad_(True)
    Y = torch.from_numpy(z["Y"]).requires_grad_(True)
    K = reference_forward({"X": X, "Y": Y}, {"gamma": float(z["gamma"])})
    K.backward(torch.from_numpy(z["G"]))
    np.testing.assert_allclose(K.detach().numpy(), z["K"], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(X.grad.numpy(), z["dX"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(Y.grad.numpy(), z["dY"], rtol=1e-5, atol=1e-6)


def test_config_superset(monkeypatch):
    import cases.rbf.config as cfg
    monkeypatch.setenv("RBF_N", "65536")
    monkeypatch.setenv("RBF_M", "8192")
    monkeypatch.setenv("RBF_D", "32")
    monkeypatch.setenv("RBF_GAMMA", str(0.5 / 32))
    monkeypatch.setenv("RBF_YDIST", "uniform")
    c = importlib.reload(cfg)
    try:
        assert (c.N, c.M, c.D, c.GAMMA, c.YDIST) == (65536, 8192, 32, 0.5 / 32, "uniform")
    finally:
        for k in ("RBF_N", "RBF_M", "RBF_D", "RBF_GAMMA", "RBF_YDIST"):
            monkeypatch.delenv(k)
        importlib.reload(cfg)


def test_configs_and_work_model():
    from cases.rbf import config
    assert set(config.CONFIGS) == {"c0", "c1", "c2", "c3", "c4"}
    c1 = config.CONFIGS["c1"]
    assert (c1["N"], c1["M"], c1["D"]) == (4096, 4096, 64)
    assert config.flops(4096, 4096, 64) == 6 * 4096 * 4096 * 64
    assert config.hbm_bytes(4096, 4096, 64) == 12 * 4096 ** 2 + 12 * 8192 * 64


def test_uniform_and_scaled_draws():
    from cases.rbf.reference import draw
    X, Y = draw(3, torch.float32, "cpu", 100, 200, 8, "uniform", 1.0)
    assert Y.min() >= -2.0 and Y.max() <= 2.0
    X2, Y2 = draw(3, torch.float32, "cpu", 100, 200, 8, "normal", 0.5)
    X3, _ = draw(3, torch.float32, "cpu", 100, 200, 8, "normal", 1.0)
    torch.testing.assert_close(X2, X3 * 0.5)
