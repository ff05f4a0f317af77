"""Shapes of the cosine-similarity case (reference ``cases/cosine_sim/config.py:1-10``).

The reference fixes N = M = 2048, D = 64, fp32, with environment overrides COS_N, COS_M, COS_D;
this module keeps those names and defaults.  eps (1e-8) is a Case parameter, as in the
reference's ``CASE.params``.
"""
import os

N = int(os.environ.get("COS_N", "2048"))
M = int(os.environ.get("COS_M", "2048"))
D = int(os.environ.get("COS_D", "64"))
EPS = 1e-8
DTYPE = "float32"


def flops(N, M, D):
    """Algorithmic FLOP of one forward + backward: 2NMD (A Bh^T) + 4NMD (dS Bh, dS^T Ah)."""
    return 6 * N * M * D


def hbm_bytes(N, M, D):
    """Algorithmic HBM bytes of one forward + backward: the forward writes S (4NM), the backward
    reads dS (4NM); plus reading A, B and writing dA, dB (and the normalised rows between)."""
    return 8 * N * M + 16 * (N + M) * D
