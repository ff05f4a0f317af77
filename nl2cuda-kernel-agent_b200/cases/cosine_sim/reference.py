"""PyTorch definition of the pairwise cosine-similarity matrix: the correctness standard.

``reference_forward`` keeps the reference's broadcast form (reference
``cases/cosine_sim/reference.py:14-21``): rows are divided by ``norm + eps``, then
``(Ah[:, None, :] * Bh[None, :, :]).sum(-1)`` is reduced over D, never written as a GEMM; the
backward is torch autograd.  ``make_inputs`` follows reference ``reference.py:24-31``: A then B
drawn with ``randn`` from one ``torch.Generator(device).manual_seed(seed)``.
"""
import torch

from cases.cosine_sim import config


def reference_forward(inputs, params):
    """inputs = {"A": [N,D], "B": [M,D]}, params = {"eps": float} -> S [N,M]."""
    A, B, eps = inputs["A"], inputs["B"], params["eps"]
    Ah = A / (A.norm(dim=-1, keepdim=True) + eps)
    Bh = B / (B.norm(dim=-1, keepdim=True) + eps)
    return (Ah.unsqueeze(1) * Bh.unsqueeze(0)).sum(dim=-1)


def make_inputs(seed, dtype, device, requires_grad=False):
    """Named inputs {"A", "B"} for ``seed`` at the configured shape."""
    g = torch.Generator(device=device).manual_seed(seed)
    A = torch.randn(config.N, config.D, dtype=dtype, device=device, generator=g)
    B = torch.randn(config.M, config.D, dtype=dtype, device=device, generator=g)
    if requires_grad:
        A.requires_grad_(True)
        B.requires_grad_(True)
    return {"A": A, "B": B}
