"""Parity of the sm_100a path (through the C ABI) with the reference's outputs and the oracle."""
import ctypes

import numpy as np
import pytest
import torch

from golden_util import load, names
from gpu_util import TOL, assert_gate, run_path, to_dev
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", names())
def test_golden_fixture(name, cuda_device):
    z = load(name)
    g = float(z["gamma"])
    K, dX, dY = run_path(z["X"], z["Y"], z["G"], g)
    assert_gate(f"{name} K", K, z["K"])
    assert_gate(f"{name} dX", dX, z["dX"])
    assert_gate(f"{name} dY", dY, z["dY"])


SHAPES = [
    (1, 1, 1, 0.5), (7, 129, 3, 0.3), (128, 128, 64, 1 / 64), (129, 257, 64, 1 / 64),
    (300, 200, 100, 0.01), (257, 130, 32, 0.5 / 32), (64, 1000, 128, 1 / 128),
    (1000, 333, 256, 1 / 256), (33, 65, 8, 0.2), (5, 3, 2048, 1 / 2048),
    # M % 4 == 0: the tensor-core backward (TMA-pitched G and K rows)
    (200, 300, 64, 1 / 64), (129, 260, 32, 0.5 / 32), (513, 1028, 64, 1 / 64), (4, 8, 3, 0.3),
    (1, 4, 1, 0.5), (700, 516, 256, 1 / 256), (300, 400, 100, 0.01), (1100, 1200, 128, 1 / 128),
    (77, 4096, 64, 1 / 64), (4096, 36, 48, 0.02),
    # M % 4 == 0 with D % 4 != 0: tensor-core backward, dX flushed with red.add; D = 130 runs two
    # 64-feature slices (G and K read twice)
    (517, 1000, 37, 1 / 37), (300, 400, 130, 1 / 130),
]


@pytest.mark.parametrize("N,M,D,gamma", SHAPES)
def test_random_shapes_vs_oracle(N, M, D, gamma, cuda_device):
    r = np.random.default_rng(N * 1000 + M + D)
    X = r.standard_normal((N, D)).astype(np.float32)
    Y = r.standard_normal((M, D)).astype(np.float32)
    G = r.standard_normal((N, M)).astype(np.float32)
    K, dX, dY = run_path(X, Y, G, gamma)
    Kr = oracle.forward(X, Y, gamma)
    dXr, dYr = oracle.backward(X, Y, G, gamma)
    assert_gate("K", K, Kr)
    assert_gate("dX", dX, dXr)
    assert_gate("dY", dY, dYr)


def test_prepared_and_shard_entries_agree(cuda_device):
    from cases.rbf import native
    r = np.random.default_rng(5)
    X, Y = r.standard_normal((300, 64)), r.standard_normal((200, 64))
    G = r.standard_normal((300, 200))
    Xd, Yd, Gd = to_dev(X, Y, G)
    K, ws = native.forward_with_workspace(Xd, Yd, 0.02)
    a = native.rbf_backward(Xd, Yd, Gd, K, 0.02, workspace=ws)
    b = native.rbf_backward(Xd, Yd, Gd, K, 0.02)
    c = native.rbf_backward(Xd, Yd, Gd, K, 0.02, entry="rbf_sm100_backward_shard")
    # The backward sums per-tile partials with fp32 atomics, so the summation order (and the
    # last bits) may differ between calls; the entries must agree to fp32 rounding.
    for u, v, w in zip(a, b, c):
        torch.testing.assert_close(u, v, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(u, w, rtol=1e-5, atol=1e-6)


def test_forward_is_deterministic(cuda_device):
    from cases.rbf import native
    Xd, Yd = to_dev(*np.random.default_rng(9).standard_normal((2, 500, 64)))
    K1 = native.rbf_forward(Xd, Yd, 1 / 64)
    K2 = native.rbf_forward(Xd, Yd, 1 / 64)
    assert torch.equal(K1, K2)


def test_noncontiguous_and_misaligned_inputs(cuda_device):
    from cases.rbf import native
    r = np.random.default_rng(2)
    big = to_dev(r.standard_normal((101, 7)))[0]
    X = big[1:]          # 28-byte offset: not 16-byte aligned, copied by the binding
    Y = to_dev(r.standard_normal((7, 50)))[0].t()   # non-contiguous
    K = native.rbf_forward(X, Y, 0.3)
    assert_gate("K", K.cpu().numpy(), oracle.forward(X.cpu().numpy(), Y.cpu().numpy(), 0.3))


def test_errors_raise(cuda_device):
    from cases.rbf import native
    X = torch.randn(4, 3, device=cuda_device)
    with pytest.raises(RuntimeError, match="share feature dim"):
        native.rbf_forward(X, torch.randn(4, 5, device=cuda_device), 0.5)
    with pytest.raises(RuntimeError, match="float32"):
        native.rbf_forward(X.double(), X.double(), 0.5)
    with pytest.raises(RuntimeError, match="not finite"):
        native.rbf_forward(X, X, float("inf"))


def test_legacy_host_pointer_abi(cuda_device):
    from cases.rbf import native
    L = native.lib()
    r = np.random.default_rng(1234)
    N, M, D, g = 128, 128, 64, 1 / 64  # the reference delivery self-test size
    X = r.uniform(-1, 1, (N, D)).astype(np.float32)
    Y = r.uniform(-1, 1, (M, D)).astype(np.float32)
    G = r.uniform(-1, 1, (N, M)).astype(np.float32)
    K = np.empty((N, M), np.float32)
    dX = np.empty((N, D), np.float32)
    dY = np.empty((M, D), np.float32)
    fp = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    L.rbf_forward_cuda.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3 + [ctypes.c_float]
    L.rbf_backward_cuda.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int] * 3 + [ctypes.c_float]
    L.rbf_forward_cuda(fp(X), fp(Y), fp(K), N, M, D, g)
    L.rbf_backward_cuda(fp(X), fp(Y), fp(G), fp(K), fp(dX), fp(dY), N, M, D, g)
    assert_gate("K", K, oracle.forward(X, Y, g))
    dXr, dYr = oracle.backward(X, Y, G, g)
    assert_gate("dX", dX, dXr)
    assert_gate("dY", dY, dYr)


def test_empty_sizes(cuda_device):
    from cases.rbf import native
    for (N, M, D) in [(0, 5, 3), (5, 0, 3), (4, 6, 0)]:
        X = torch.randn(N, D, device=cuda_device)
        Y = torch.randn(M, D, device=cuda_device)
        G = torch.randn(N, M, device=cuda_device)
        K, ws = native.forward_with_workspace(X, Y, 0.5)
        dX, dY = native.rbf_backward(X, Y, G, K, 0.5, workspace=ws)
        assert K.shape == (N, M) and dX.shape == (N, D) and dY.shape == (M, D)
        if N and M:
            assert torch.all(K == 1.0)  # D = 0: distance 0
        assert torch.all(dX == 0) and torch.all(dY == 0)


PAIR_SHAPES = [(1, 4, 1, 0.5), (129, 260, 32, 0.5 / 32), (257, 128, 64, 1 / 64),
               (300, 516, 48, 0.02), (513, 1028, 64, 1 / 64), (4096, 4096, 64, 1 / 64)]


@pytest.mark.parametrize("N,M,D,gamma", PAIR_SHAPES)
def test_forward_pair_and_single_cta_variants(N, M, D, gamma, cuda_device, monkeypatch):
    """D <= 64 with M % 4 == 0: RBF_FWD_PAIR=1 runs the two-CTA (cta_group::2) forward, 0 (the
    default) single-CTA tiles.  Both must meet the gate against the oracle."""
    from cases.rbf import native
    r = np.random.default_rng(N + 7 * M + 13 * D)
    X = r.standard_normal((N, D)).astype(np.float32)
    Y = r.standard_normal((M, D)).astype(np.float32)
    Xd, Yd = to_dev(X, Y)
    rows = np.unique(np.linspace(0, N - 1, min(N, 256)).astype(np.int64))
    Kr = oracle.forward(X[rows], Y, gamma)
    out = {}
    for flag in ("1", "0"):
        monkeypatch.setenv("RBF_FWD_PAIR", flag)
        K = native.rbf_forward(Xd, Yd, gamma)
        torch.cuda.synchronize()
        out[flag] = K.cpu().numpy()
        assert_gate(f"K pair={flag}", out[flag][rows], Kr)
    np.testing.assert_allclose(out["1"], out["0"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("N,M,D,gamma", [(300, 200, 64, 0.02), (517, 1000, 37, 1 / 37),
                                         (129, 260, 32, 0.5 / 32), (7, 129, 3, 0.3),
                                         (1000, 333, 256, 1 / 256)])
def test_forward_backward_entry(N, M, D, gamma, cuda_device):
    """rbf_sm100_forward_backward: the two-call path's K, dX, dY, and the oracle's."""
    from cases.rbf import native
    r = np.random.default_rng(N + 7 * M + D)
    X = r.standard_normal((N, D)).astype(np.float32)
    Y = r.standard_normal((M, D)).astype(np.float32)
    G = r.standard_normal((N, M)).astype(np.float32)
    Xd, Yd, Gd = to_dev(X, Y, G)
    K, dX, dY = native.rbf_forward_backward(Xd, Yd, Gd, gamma)
    K2, ws = native.forward_with_workspace(Xd, Yd, gamma)
    dX2, dY2 = native.rbf_backward(Xd, Yd, Gd, K2, gamma, workspace=ws)
    assert torch.equal(K, K2)
    # The backward's atomic flushes add in a run-dependent fp32 order.
    torch.testing.assert_close(dX, dX2, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(dY, dY2, rtol=1e-4, atol=1e-4)
    assert_gate("K", K.cpu().numpy(), oracle.forward(X, Y, gamma))
    dXr, dYr = oracle.backward(X, Y, G, gamma)
    assert_gate("dX", dX.cpu().numpy(), dXr)
    assert_gate("dY", dY.cpu().numpy(), dYr)


def test_forward_backward_entry_refuses_the_forward_workspace(cuda_device):
    from cases.rbf import native
    L = native.lib()
    X = torch.randn(64, 64, device="cuda")
    G = torch.randn(64, 64, device="cuda")
    K = torch.full((64, 64), 7.0, device="cuda")
    dX, dY = torch.empty(64, 64, device="cuda"), torch.empty(64, 64, device="cuda")
    small = L.rbf_sm100_forward_workspace_bytes(64, 64, 64)
    assert small < L.rbf_sm100_backward_workspace_bytes(64, 64, 64)
    ws = torch.empty(small, dtype=torch.uint8, device="cuda")
    vp = ctypes.c_void_p
    st = L.rbf_sm100_forward_backward(vp(X.data_ptr()), vp(X.data_ptr()), vp(G.data_ptr()),
                                      vp(K.data_ptr()), vp(dX.data_ptr()), vp(dY.data_ptr()),
                                      64, 64, 64, 0.1, vp(ws.data_ptr()), small,
                                      vp(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert st == 3  # RBF_ERR_WORKSPACE
    assert bool((K == 7.0).all())  # refused before the forward ran


def test_underflowing_kernel_values_vs_oracle(cuda_device):
    """gamma * ||x - y||^2 from about 1 to 250: K runs from 0.3 through the subnormal range
    (below 1.2e-38, 5 % of the entries) down to 0.  The exp path flushes results below 2^-126 to
    zero; that and the matching dX / dY terms stay inside the 1e-3 gate."""
    r = np.random.default_rng(17)
    N, M, D = 256, 300, 64
    X = r.standard_normal((N, D)).astype(np.float32)
    Y = np.concatenate([X[:100] + 0.3 * r.standard_normal((100, D)),
                        2.0 * r.standard_normal((200, D)) + 1.0]).astype(np.float32)
    gamma = 0.35
    G = r.standard_normal((N, M)).astype(np.float32)
    K, dX, dY = run_path(X, Y, G, gamma)
    Kr = oracle.forward(X, Y, gamma)
    assert ((Kr > 1e-45) & (Kr < 1.2e-38)).mean() > 0.02 and (Kr > 1e-6).any()
    assert_gate("K", K, Kr)
    dXr, dYr = oracle.backward(X, Y, G, gamma)
    assert_gate("dX", dX, dXr)
    assert_gate("dY", dY, dYr)
    assert np.isfinite(K).all() and (K >= 0).all()
