"""Parity of the cosine-similarity path (tcgen05 forward / backward in their DOT instantiations,
through the cos_sm100_* C ABI) with the reference's own outputs and the fp64 oracle."""
import numpy as np
import pytest
import torch

from golden_util import cos_names, load
from gpu_util import assert_gate, to_dev
from oracle import cos_oracle

pytestmark = pytest.mark.gpu

EPS = 1e-8


def run_cos(A, B, dS, eps=EPS, prepared=True):
    """Forward + backward through the C ABI -> numpy (S, dA, dB)."""
    from cases.cosine_sim import native
    Ad, Bd, dSd = to_dev(A, B, dS)
    N, D = Ad.shape
    M = Bd.size(0)
    S, ws = native.forward_with_workspace(Ad, Bd, eps)
    if prepared:
        dA, dB = native.cos_backward(dSd, N, M, D, eps, workspace=ws)
    else:
        dA, dB = native.cos_backward(dSd, N, M, D, eps, A=Ad, B=Bd)
    torch.cuda.synchronize()
    return S.cpu().numpy(), dA.cpu().numpy(), dB.cpu().numpy()


def assert_close_to(name, got, ref, tight=1e-4):
    """The 1e-3 gate of the path, and a tighter bound relative to the largest value: 3xTF32
    keeps fp32-level accuracy, so errors far above fp32 rounding mean a broken kernel.  (At
    D = 1 the gradients are 0 up to rounding -- a row's gradient is orthogonal to the row -- so
    only the gate applies; tight=None.)"""
    assert_gate(name, got, ref)
    if tight is not None and np.size(ref):
        scale = float(np.max(np.abs(ref)))
        err = float(np.max(np.abs(np.asarray(got, np.float64) - ref)))
        assert err <= tight * max(scale, 1e-30), (name, err, scale)


@pytest.mark.parametrize("name", cos_names())
@pytest.mark.parametrize("prepared", [True, False])
def test_golden_fixture(name, prepared, cuda_device):
    z = load(name)
    S, dA, dB = run_cos(z["A"], z["B"], z["dS"], float(z["eps"]), prepared)
    tight = 1e-4 if z["A"].shape[1] > 1 else None
    assert_close_to(f"{name} S", S, z["S"])
    assert_close_to(f"{name} dA", dA, z["dA"], tight)
    assert_close_to(f"{name} dB", dB, z["dB"], tight)


SHAPES = [
    (1, 4, 1), (128, 128, 64), (2048, 2048, 64), (300, 200, 100), (1000, 332, 256),
    (517, 1000, 37), (77, 4096, 64), (4096, 36, 48), (5, 8, 2048), (129, 260, 32),
    # M % 4 != 0: the CUDA-core backward reads the normalised rows from the workspace
    (129, 257, 64), (33, 65, 8), (300, 201, 130),
]


@pytest.mark.parametrize("N,M,D", SHAPES)
def test_random_shapes_vs_oracle(N, M, D, cuda_device):
    r = np.random.default_rng(N * 7919 + M * 31 + D)
    A = r.standard_normal((N, D)).astype(np.float32)
    B = (3.0 * r.standard_normal((M, D))).astype(np.float32)
    dS = r.standard_normal((N, M)).astype(np.float32)
    S, dA, dB = run_cos(A, B, dS)
    assert_close_to("S", S, cos_oracle.forward(A, B, EPS))
    dAr, dBr = cos_oracle.backward(A, B, dS, EPS)
    tight = 1e-4 if D > 1 else None
    assert_close_to("dA", dA, dAr, tight)
    assert_close_to("dB", dB, dBr, tight)


def test_verify_all_passes(cuda_device):
    from cases.cosine_sim import CASE
    from cases.cosine_sim.op import candidate
    from framework.verify import verify_all
    ok, report = verify_all(CASE, candidate, device="cuda")
    print(report)
    assert ok, report


def test_candidate_within_1e3_of_reference(cuda_device):
    from cases.cosine_sim import CASE
    from cases.cosine_sim.op import candidate, forward_only
    base = CASE.make_inputs(3, torch.float32, "cuda")
    ref = {k: v.clone().requires_grad_(True) for k, v in base.items()}
    imp = {k: v.clone().requires_grad_(True) for k, v in base.items()}
    Sr = CASE.reference_forward(ref, CASE.params)
    dS = torch.randn(Sr.shape, device="cuda",
                     generator=torch.Generator(device="cuda").manual_seed(10_003))
    Sr.backward(dS)
    Si = candidate(imp, CASE.params)
    Si.backward(dS)
    for a, b in ((Si, Sr), (imp["A"].grad, ref["A"].grad), (imp["B"].grad, ref["B"].grad)):
        torch.testing.assert_close(a.detach(), b.detach(), atol=1e-3, rtol=1e-3)
    torch.testing.assert_close(forward_only(base, CASE.params), Sr.detach(), atol=1e-3,
                               rtol=1e-3)


def test_large_size_properties(cuda_device):
    """N = M = 8192: S of A with itself is symmetric with a unit diagonal; sampled rows of S
    and dA, and all of dB, against the fp64 oracle."""
    from cases.cosine_sim import native
    r = np.random.default_rng(17)
    N, D = 8192, 64
    A = r.standard_normal((N, D)).astype(np.float32)
    dS = r.standard_normal((N, N)).astype(np.float32)
    Ad, dSd = to_dev(A, dS)
    S, ws = native.forward_with_workspace(Ad, Ad, EPS)
    dA, dB = native.cos_backward(dSd, N, N, D, EPS, workspace=ws)
    torch.cuda.synchronize()
    diag = torch.diagonal(S)
    assert float((diag - 1).abs().max()) < 1e-5
    assert float((S - S.T).abs().max()) < 1e-5
    assert float(S.abs().max()) <= 1 + 1e-5
    rows = np.array([0, 1, 4095, 8191, 777])
    assert_close_to("S rows", S[rows].cpu().numpy(), cos_oracle.forward(A[rows], A, EPS))
    dAr, dBr = cos_oracle.backward(A, A, dS, EPS)
    assert_close_to("dA", dA.cpu().numpy(), dAr)
    assert_close_to("dB", dB.cpu().numpy(), dBr)


def test_backward_entries_agree_and_forward_is_deterministic(cuda_device):
    from cases.cosine_sim import native
    r = np.random.default_rng(3)
    A, B, dS = (r.standard_normal(s).astype(np.float32) for s in ((300, 64), (200, 64), (300, 200)))
    Ad, Bd, dSd = to_dev(A, B, dS)
    S1, ws = native.forward_with_workspace(Ad, Bd, EPS)
    S2 = native.cos_forward(Ad, Bd, EPS)
    assert torch.equal(S1, S2)
    a = native.cos_backward(dSd, 300, 200, 64, EPS, workspace=ws)
    b = native.cos_backward(dSd, 300, 200, 64, EPS, A=Ad, B=Bd)
    for u, v in zip(a, b):
        torch.testing.assert_close(u, v, rtol=1e-5, atol=1e-6)


def test_errors_raise(cuda_device):
    from cases.cosine_sim import native
    A = torch.randn(4, 8, device="cuda")
    with pytest.raises(RuntimeError, match="feature dim"):
        native.cos_forward(A, torch.randn(4, 9, device="cuda"), EPS)
    with pytest.raises(RuntimeError, match="eps"):
        native.cos_forward(A, A, float("nan"))
    with pytest.raises(RuntimeError, match="shape"):
        native.cos_backward(torch.randn(3, 4, device="cuda"), 4, 4, 8, EPS, A=A, B=A)
