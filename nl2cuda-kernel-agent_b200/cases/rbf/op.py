"""The RBF candidate: autograd op over the sm_100a kernels (reference ``cases/rbf/op.py:17-49``).

``candidate(inputs, params) -> K`` is the harness contract; gradients flow to ``inputs["X"]``
and ``inputs["Y"]``.  As in the reference, the forward saves X, Y and K for the backward; it
also saves the workspace holding the TF32 split of X and Y, so the backward skips that pass.
"""
import torch

from cases.rbf import native, shard


class RBFFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, X, Y, gamma):
        K, ws = native.forward_with_workspace(X, Y, float(gamma))
        ctx.save_for_backward(X, Y, K)
        ctx.workspace = ws
        ctx.gamma = float(gamma)
        return K

    @staticmethod
    def backward(ctx, G):
        X, Y, K = ctx.saved_tensors
        dX, dY = native.rbf_backward(X, Y, G.contiguous(), K, ctx.gamma, workspace=ctx.workspace)
        if shard.check_status_default():
            # RBF_CHECK_STATUS=1: one synchronisation per step, so that a bounded device wait
            # that ran out (in the forward or this backward) raises instead of returning partial
            # gradients.
            st = native.read_status(ctx.workspace)
            if st != 0:
                raise RuntimeError(f"rbf backward: device status {st} (a bounded device-side "
                                   "wait timed out)")
        ctx.workspace = None
        return dX, dY, None


def candidate(inputs, params):
    """Harness contract: inputs = {"X", "Y"}, params = {"gamma"} -> K."""
    return RBFFunction.apply(inputs["X"], inputs["Y"], params["gamma"])


def forward_only(inputs, params):
    """Forward without autograd (reference op.py:47-49)."""
    return native.rbf_forward(inputs["X"], inputs["Y"], float(params["gamma"]))
