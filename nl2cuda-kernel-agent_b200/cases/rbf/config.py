"""Shapes and scalar parameters of the RBF case (reference ``cases/rbf/config.py:11-17``).

The reference fixes N = M = ``RBF_SIZE`` (default 2048), D = 64, gamma = 1/64, fp32.  This
module keeps those defaults and names, and adds environment overrides so that every BASELINE
configuration is reachable without changing the Case protocol:

  RBF_N, RBF_M      rows of X / Y           (default RBF_SIZE)
  RBF_D             features                (default 64)
  RBF_GAMMA         gamma                   (default 1/64 when D = 64, else 1/D)
  RBF_YDIST         "normal" | "uniform"    Y ~ N(0,1) or U(-2, 2)   (default normal)
  RBF_XSCALE        multiplier of X and Y   (default 1; 1/sqrt(2) for the c4 regime)

``CONFIGS`` names the five BASELINE configurations c0-c4.
"""
import math
import os

_SIZE = int(os.environ.get("RBF_SIZE", "2048"))

N = int(os.environ.get("RBF_N", _SIZE))
M = int(os.environ.get("RBF_M", _SIZE))
D = int(os.environ.get("RBF_D", "64"))
GAMMA = float(os.environ.get("RBF_GAMMA", 1.0 / 64.0 if D == 64 else 1.0 / max(D, 1)))
YDIST = os.environ.get("RBF_YDIST", "normal")
XSCALE = float(os.environ.get("RBF_XSCALE", "1.0"))
DTYPE = "float32"

if YDIST not in ("normal", "uniform"):
    raise ValueError(f"RBF_YDIST must be 'normal' or 'uniform', not {YDIST!r}")

# The five BASELINE configurations (X, Y, G fp32; G ~ N(0,1) from an independent stream).
CONFIGS = {
    "c0": dict(N=2048, M=2048, D=64, gamma=1 / 64, ydist="normal", xscale=1.0),
    "c1": dict(N=4096, M=4096, D=64, gamma=1 / 64, ydist="normal", xscale=1.0),
    "c2": dict(N=16384, M=16384, D=128, gamma=1 / 128, ydist="normal", xscale=1.0),
    "c3": dict(N=65536, M=8192, D=32, gamma=0.5 / 32, ydist="uniform", xscale=1.0),
    "c4": dict(N=65536, M=65536, D=256, gamma=1 / 256, ydist="normal",
               xscale=1 / math.sqrt(2.0)),
}


def flops(N, M, D):
    """Algorithmic FLOP of one forward + backward: 2NMD (forward -2XY^T) + 4NMD (W Y, W^T X)."""
    return 6 * N * M * D


def hbm_bytes(N, M, D):
    """Algorithmic HBM bytes of one forward + backward: forward writes K (4NM) and reads X, Y;
    backward reads G and K (8NM), reads X, Y and writes dX, dY."""
    return 12 * N * M + 12 * (N + M) * D
