"""Parity at the full BASELINE sizes (configs c1-c4) on sampled rows and columns, plus
size-independent properties of the full outputs.

The oracle needs only the sampled slices: K[i,:] and dX[i,:] depend on x_i, Y and G[i,:];
dY[j,:] on X, y_j and G[:,j].  Property: K depends on x - y only, so the exact gradients satisfy
sum_i dX[i] + sum_j dY[j] = 0; the test bounds the fp32 residual relative to the gradients'
magnitude.
"""
import numpy as np
import pytest
import torch

from gpu_util import assert_gate
from oracle import oracle

pytestmark = pytest.mark.gpu


def _run(cfg_name, n_sample=24, seed=11):
    from cases.rbf import config, native
    from cases.rbf.reference import draw
    c = config.CONFIGS[cfg_name]
    N, M, D, g = c["N"], c["M"], c["D"], c["gamma"]
    X, Y = draw(seed, torch.float32, "cuda", N, M, D, c["ydist"], c["xscale"])
    G = torch.randn(N, M, device="cuda", generator=torch.Generator(device="cuda").manual_seed(seed))
    K, ws = native.forward_with_workspace(X, Y, g)
    dX, dY = native.rbf_backward(X, Y, G, K, g, workspace=ws)
    torch.cuda.synchronize()
    assert native.read_status(ws) == 0
    r = np.random.default_rng(seed)
    rows = np.unique(np.concatenate([[0, N - 1], r.integers(0, N, n_sample)]))
    cols = np.unique(np.concatenate([[0, M - 1], r.integers(0, M, n_sample)]))
    Xh, Yh = X.cpu().numpy(), Y.cpu().numpy()
    ri, ci = torch.from_numpy(rows).cuda(), torch.from_numpy(cols).cuda()
    Grow = G.index_select(0, ri).cpu().numpy()
    Gcol = G.index_select(1, ci).cpu().numpy()
    assert_gate(f"{cfg_name} K rows", K.index_select(0, ri).cpu().numpy(),
                oracle.forward_rows(Xh, Yh, g, rows))
    assert_gate(f"{cfg_name} dX rows", dX.index_select(0, ri).cpu().numpy(),
                oracle.dx_rows(Xh[rows], Yh, Grow, g, np.arange(len(rows))))
    assert_gate(f"{cfg_name} dY cols", dY.index_select(0, ci).cpu().numpy(),
                oracle.dy_cols(Xh, Yh[cols], Gcol, g, np.arange(len(cols))))
    # Translation invariance, in fp64 over the full outputs.
    s = dX.double().sum(0) + dY.double().sum(0)
    scale = dX.double().abs().sum(0) + dY.double().abs().sum(0)
    assert float((s.abs() / scale).max()) < 1e-4
    assert float(K.min()) >= 0.0 and float(K.max()) <= 1.0
    assert torch.isfinite(dX).all() and torch.isfinite(dY).all()


@pytest.mark.parametrize("cfg", ["c1", "c2", "c3"])
def test_config_full_size(cfg, cuda_device):
    _run(cfg)


@pytest.mark.slow
def test_config_c4_full_size(cuda_device):
    _run("c4", n_sample=8)


def test_self_kernel_is_symmetric(cuda_device):
    from cases.rbf import native
    X = torch.randn(1000, 64, device="cuda")
    K = native.rbf_forward(X, X, 1 / 64)
    torch.testing.assert_close(K, K.t(), atol=2e-6, rtol=1e-5)
    assert torch.allclose(K.diagonal(), torch.ones(1000, device="cuda"), atol=1e-5)


def test_backward_is_linear_in_g(cuda_device):
    from cases.rbf import native
    gen = torch.Generator(device="cuda").manual_seed(3)
    X = torch.randn(700, 64, device="cuda", generator=gen)
    Y = torch.randn(900, 64, device="cuda", generator=gen)
    G1 = torch.randn(700, 900, device="cuda", generator=gen)
    G2 = torch.randn(700, 900, device="cuda", generator=gen)
    K, ws = native.forward_with_workspace(X, Y, 1 / 64)
    a = native.rbf_backward(X, Y, G1, K, 1 / 64, workspace=ws)
    b = native.rbf_backward(X, Y, G2, K, 1 / 64, workspace=ws)
    c = native.rbf_backward(X, Y, G1 + 2 * G2, K, 1 / 64, workspace=ws)
    for u, v, w in zip(a, b, c):
        torch.testing.assert_close(w, u + 2 * v, atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("case", ["rbf", "cosine_sim"])
def test_backward_repeatable_at_8192(case, cuda_device):
    """30 backward passes at N = M = 8192 agree with the first to fp32 rounding (the atomic
    flushes reorder sums, nothing more).  Guards the pipeline's buffer hand-offs: a stage reused
    before every lane had read it showed up here as a wrong block of rows in a few runs of 30."""
    from cases.cosine_sim import native as cn
    from cases.rbf import native
    gen = torch.Generator(device="cuda").manual_seed(8192)
    N = M = 8192
    X = torch.randn(N, 64, device="cuda", generator=gen)
    Y = torch.randn(M, 64, device="cuda", generator=gen)
    G = torch.randn(N, M, device="cuda", generator=gen)
    if case == "rbf":
        K, ws = native.forward_with_workspace(X, Y, 1 / 64)
        run = lambda: native.rbf_backward(X, Y, G, K, 1 / 64, workspace=ws)  # noqa: E731
    else:
        _, ws = cn.forward_with_workspace(X, Y, 1e-8)
        run = lambda: cn.cos_backward(G, N, M, 64, 1e-8, workspace=ws)  # noqa: E731
    first = [t.clone() for t in run()]
    for _ in range(30):
        for u, v in zip(run(), first):
            torch.testing.assert_close(u, v, rtol=1e-4, atol=1e-5)
    assert native.read_status(ws) == 0
