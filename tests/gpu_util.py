"""Helpers of the GPU parity tests: run the sm_100a path through the C ABI and compare with the
oracle under the 1e-3 gate."""
import numpy as np
import torch

from oracle import oracle

# max abs/rel error 1e-3 vs the reference, as an allclose-style gate
# |got - ref| <= TOL + TOL * |ref|.
TOL = 1e-3


def to_dev(*arrays, device="cuda:0"):
    return [torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(device) for a in arrays]


def run_path(X, Y, G, gamma):
    """Forward + prepared backward through the C ABI -> numpy (K, dX, dY)."""
    from cases.rbf import native
    Xd, Yd, Gd = to_dev(X, Y, G)
    K, ws = native.forward_with_workspace(Xd, Yd, gamma)
    dX, dY = native.rbf_backward(Xd, Yd, Gd, K, gamma, workspace=ws)
    torch.cuda.synchronize()
    return K.cpu().numpy(), dX.cpu().numpy(), dY.cpu().numpy()


def assert_gate(name, got, ref, tol=TOL):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, (name, got.shape, ref.shape)
    if ref.size == 0:
        return
    bad = np.abs(got - ref) > tol + tol * np.abs(ref)
    if bad.any():
        idx = np.unravel_index(np.argmax(np.abs(got - ref)), ref.shape)
        raise AssertionError(f"{name}: {int(bad.sum())} of {ref.size} elements outside the "
                             f"{tol} gate; worst at {idx}: got {got[idx]!r} ref {ref[idx]!r}")
