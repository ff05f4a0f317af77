"""The harness gates of the reference (5-seed allclose(1e-2) forward + backward) on the
sm_100a candidate, and the 1e-3 gate against the broadcast reference on the same device."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_verify_all_passes(cuda_device):
    from cases.rbf import CASE
    from cases.rbf.op import candidate
    from framework.verify import verify_all
    ok, report = verify_all(CASE, candidate, device="cuda")
    print(report)
    assert ok, report


def test_candidate_within_1e3_of_reference_all_seeds(cuda_device):
    from cases.rbf import CASE
    from cases.rbf.op import candidate
    for seed in range(5):
        base = CASE.make_inputs(seed, torch.float32, "cuda")
        ref = {k: v.clone().requires_grad_(True) for k, v in base.items()}
        imp = {k: v.clone().requires_grad_(True) for k, v in base.items()}
        Kr = CASE.reference_forward(ref, CASE.params)
        G = torch.randn(Kr.shape, device="cuda",
                        generator=torch.Generator(device="cuda").manual_seed(seed + 10_000))
        Kr.backward(G)
        Ki = candidate(imp, CASE.params)
        Ki.backward(G)
        for a, b in ((Ki, Kr), (imp["X"].grad, ref["X"].grad), (imp["Y"].grad, ref["Y"].grad)):
            torch.testing.assert_close(a.detach(), b.detach(), atol=1e-3, rtol=1e-3)


def test_forward_only(cuda_device):
    from cases.rbf import CASE
    from cases.rbf.op import forward_only
    inp = CASE.make_inputs(0, torch.float32, "cuda")
    torch.testing.assert_close(forward_only(inp, CASE.params),
                               CASE.reference_forward(inp, CASE.params), atol=1e-3, rtol=1e-3)
