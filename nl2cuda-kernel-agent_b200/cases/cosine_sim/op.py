"""The cosine-similarity candidate: autograd op over the sm_100a kernels (reference
``cases/cosine_sim/op.py:18-42``).

``candidate(inputs, params) -> S`` is the harness contract; gradients flow to ``inputs["A"]`` and
``inputs["B"]``.  Where the reference's forward saves Ah, Bh, invA, invB for the backward, this
one saves the workspace that holds the normalised rows (TF32 hi/lo) and the norms.
"""
import torch

from cases.cosine_sim import native


class CosineSimFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, A, B, eps):
        S, ws = native.forward_with_workspace(A, B, float(eps))
        ctx.workspace = ws
        ctx.shape = (A.size(0), B.size(0), A.size(1))
        ctx.eps = float(eps)
        return S

    @staticmethod
    def backward(ctx, dS):
        N, M, D = ctx.shape
        dA, dB = native.cos_backward(dS.contiguous(), N, M, D, ctx.eps, workspace=ctx.workspace)
        ctx.workspace = None
        return dA, dB, None


def candidate(inputs, params):
    """Harness contract: inputs = {"A", "B"}, params = {"eps"} -> S."""
    return CosineSimFunction.apply(inputs["A"], inputs["B"], params["eps"])


def forward_only(inputs, params):
    """Forward without autograd (reference op.py:39-42)."""
    return native.cos_forward(inputs["A"], inputs["B"], float(params["eps"]))
