"""RBF_DETERMINISTIC=1: the backward stores each tile's partials into its own workspace slot and
sums them in a fixed order, so dX and dY are bit-identical from run to run.  Checked at 8192²
(10 runs, torch.equal), against the oracle, against the default (atomic) mode, on ragged shapes
and for the cosine backward, which shares the kernel."""
import numpy as np
import pytest
import torch

from gpu_util import assert_gate, to_dev
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture
def deterministic(monkeypatch):
    monkeypatch.setenv("RBF_DETERMINISTIC", "1")


def _backward(X, Y, G, g):
    from cases.rbf import native
    K, ws = native.forward_with_workspace(X, Y, g)
    dX, dY = native.rbf_backward(X, Y, G, K, g, workspace=ws)
    torch.cuda.synchronize()
    assert native.read_status(ws) == 0
    return dX, dY


def test_backward_bit_identical_at_8192(cuda_device, monkeypatch):
    N = M = 8192
    D, g = 64, 1 / 64
    gen = torch.Generator(device="cuda").manual_seed(3)
    X = torch.randn(N, D, device="cuda", generator=gen)
    Y = torch.randn(M, D, device="cuda", generator=gen)
    G = torch.randn(N, M, device="cuda", generator=gen)
    dflt = _backward(X, Y, G, g)
    monkeypatch.setenv("RBF_DETERMINISTIC", "1")
    first = _backward(X, Y, G, g)
    for _ in range(9):
        dX, dY = _backward(X, Y, G, g)
        assert torch.equal(dX, first[0]) and torch.equal(dY, first[1])
    # The default mode adds the same partials atomically, in a run-dependent fp32 order: dY sums
    # 8192 products, so the two agree to fp32 rounding of such sums, not bit for bit.
    torch.testing.assert_close(dflt[0], first[0], rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(dflt[1], first[1], rtol=1e-4, atol=1e-4)
    # Oracle on sampled rows and columns.
    r = np.random.default_rng(0)
    rows = np.unique(np.concatenate([[0, N - 1], r.integers(0, N, 12)]))
    cols = np.unique(np.concatenate([[0, M - 1], r.integers(0, M, 12)]))
    Xh, Yh = X.cpu().numpy(), Y.cpu().numpy()
    ri, ci = torch.from_numpy(rows).cuda(), torch.from_numpy(cols).cuda()
    assert_gate("dX rows", first[0].index_select(0, ri).cpu().numpy(),
                oracle.dx_rows(Xh[rows], Yh, G.index_select(0, ri).cpu().numpy(), g,
                               np.arange(len(rows))))
    assert_gate("dY cols", first[1].index_select(0, ci).cpu().numpy(),
                oracle.dy_cols(Xh, Yh[cols], G.index_select(1, ci).cpu().numpy(), g,
                               np.arange(len(cols))))


@pytest.mark.parametrize("N,M,D,gamma", [(300, 400, 130, 1 / 130), (517, 1000, 37, 1 / 37),
                                         (129, 260, 32, 0.5 / 32), (1, 4, 1, 0.5)])
def test_ragged_shapes_vs_oracle(N, M, D, gamma, cuda_device, deterministic):
    r = np.random.default_rng(N + M + D)
    X = r.standard_normal((N, D)).astype(np.float32)
    Y = r.standard_normal((M, D)).astype(np.float32)
    G = r.standard_normal((N, M)).astype(np.float32)
    Xd, Yd, Gd = to_dev(X, Y, G)
    a = _backward(Xd, Yd, Gd, gamma)
    b = _backward(Xd, Yd, Gd, gamma)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    dXr, dYr = oracle.backward(X, Y, G, gamma)
    assert_gate("dX", a[0].cpu().numpy(), dXr)
    assert_gate("dY", a[1].cpu().numpy(), dYr)


def test_cosine_backward_bit_identical(cuda_device, deterministic):
    from cases.cosine_sim import native as cn
    N = M = 4096
    D = 64
    gen = torch.Generator(device="cuda").manual_seed(5)
    A = torch.randn(N, D, device="cuda", generator=gen)
    B = torch.randn(M, D, device="cuda", generator=gen)
    dS = torch.randn(N, M, device="cuda", generator=gen)
    outs = []
    for _ in range(5):
        _, ws = cn.forward_with_workspace(A, B, 1e-8)
        outs.append(cn.cos_backward(dS, N, M, D, 1e-8, workspace=ws))
    torch.cuda.synchronize()
    for o in outs[1:]:
        assert all(torch.equal(x, y) for x, y in zip(o, outs[0]))
