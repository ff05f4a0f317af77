"""PyTorch definition of the RBF kernel matrix: the correctness standard of the Case.

``reference_forward`` is the reference's broadcast form (reference ``cases/rbf/reference.py:14-20``):
it materialises ``X[:,None,:] - Y[None,:,:]`` ([N, M, D]) and reduces it, never the
``||x||^2 + ||y||^2 - 2 X Y^T`` expansion; its backward is torch autograd.
``make_inputs`` follows reference ``reference.py:23-31``: X then Y drawn with ``randn`` from one
``torch.Generator(device).manual_seed(seed)``; with the default config it yields the same
tensors as the reference (pinned by tests/test_case_surface.py against golden fixtures).  The
extra config knobs (RBF_YDIST, RBF_XSCALE) reshape the distributions for configs c3 and c4.
"""
import torch

from cases.rbf import config


def reference_forward(inputs, params):
    """inputs = {"X": [N,D], "Y": [M,D]}, params = {"gamma": float} -> K [N,M]."""
    X, Y = inputs["X"], inputs["Y"]
    diff = X.unsqueeze(1) - Y.unsqueeze(0)
    return torch.exp(-params["gamma"] * diff.pow(2).sum(dim=-1))


def draw(seed, dtype, device, N, M, D, ydist="normal", xscale=1.0):
    """X [N,D] then Y [M,D] from one generator seeded with ``seed`` on ``device``."""
    g = torch.Generator(device=device).manual_seed(seed)
    X = torch.randn(N, D, dtype=dtype, device=device, generator=g)
    if ydist == "uniform":
        Y = torch.rand(M, D, dtype=dtype, device=device, generator=g) * 4.0 - 2.0
    else:
        Y = torch.randn(M, D, dtype=dtype, device=device, generator=g)
    if xscale != 1.0:
        X = X * xscale
        Y = Y * xscale
    return X, Y


def make_inputs(seed, dtype, device, requires_grad=False):
    """Named inputs {"X", "Y"} for ``seed`` at the configured shape."""
    X, Y = draw(seed, dtype, device, config.N, config.M, config.D, config.YDIST, config.XSCALE)
    if requires_grad:
        X.requires_grad_(True)
        Y.requires_grad_(True)
    return {"X": X, "Y": Y}
