"""Generate the golden fixtures in this directory from the reference's own RBF code.

Runs the reference project's ``cases/rbf/reference.py`` (``reference_forward`` and
``make_inputs``) with torch on the CPU, plus torch autograd for the backward, exactly as the
reference's ``framework/verify.py`` does (G drawn from ``torch.Generator().manual_seed(seed +
10000)``, ``verify.py:62``).  The reference is imported from the path given by ``--reference``
(default: the environment variable RBF_REFERENCE_ROOT); it is only needed to regenerate the
fixtures, never to run the tests.

Usage:  python tests/golden/make_golden.py --reference <path-to-reference-checkout>
"""
import argparse
import importlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(root, size):
    os.environ["RBF_SIZE"] = str(size)
    if root not in sys.path:
        sys.path.insert(0, root)
    for m in [m for m in list(sys.modules) if m == "cases" or m.startswith("cases.")
              or m == "framework" or m.startswith("framework.")]:
        del sys.modules[m]
    config = importlib.import_module("cases.rbf.config")
    reference = importlib.import_module("cases.rbf.reference")
    return config, reference


def _run(reference, X, Y, gamma, G):
    Xr = X.clone().requires_grad_(True)
    Yr = Y.clone().requires_grad_(True)
    K = reference.reference_forward({"X": Xr, "Y": Yr}, {"gamma": gamma})
    K.backward(G)
    return K.detach(), Xr.grad.detach(), Yr.grad.detach()


def _save(name, X, Y, G, gamma, K, dX, dY, note):
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, X=X.numpy(), Y=Y.numpy(), G=G.numpy(), gamma=np.float64(gamma),
                        K=K.numpy(), dX=dX.numpy(), dY=dY.numpy(), note=np.array(note))
    print(f"wrote {path}  X{tuple(X.shape)} Y{tuple(Y.shape)} gamma={gamma:.6g}  ({note})")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("RBF_REFERENCE_ROOT"))
    args = ap.parse_args()
    if not args.reference:
        raise SystemExit("pass --reference <reference checkout> or set RBF_REFERENCE_ROOT")
    torch.manual_seed(0)

    # 1) The reference's own input generator and verify.py's G stream: the 5-seed gate at a
    #    size the CPU finishes quickly.  Seed 0 at N=M=128 (the delivery self-test size,
    #    delivery/rbf_test.cu:67), seeds 1-4 at N=M=64.
    for seed, size in [(0, 128), (1, 64), (2, 64), (3, 64), (4, 64)]:
        config, reference = _import_reference(args.reference, size)
        inp = reference.make_inputs(seed, torch.float32, "cpu")
        X, Y = inp["X"], inp["Y"]
        g = torch.Generator(device="cpu").manual_seed(seed + 10_000)
        K0 = reference.reference_forward(inp, {"gamma": config.GAMMA})
        G = torch.randn(K0.shape, dtype=torch.float32, device="cpu", generator=g)
        K, dX, dY = _run(reference, X, Y, config.GAMMA, G)
        _save(f"ref_makeinputs_seed{seed}_n{size}", X, Y, G, config.GAMMA, K, dX, dY,
              f"reference make_inputs(seed={seed}) RBF_SIZE={size}; G seed {seed + 10000}")

    config, reference = _import_reference(args.reference, 64)
    gen = torch.Generator().manual_seed(1234)

    def randn(*s):
        return torch.randn(*s, generator=gen, dtype=torch.float32)

    # 2) Ragged, odd D, not a multiple of any tile.
    X, Y = randn(37, 5), randn(50, 5)
    G = randn(37, 50)
    _save("ragged_n37_m50_d5", X, Y, G, 0.2, *_run(reference, X, Y, 0.2, G), "ragged odd D")

    # 3) The c3 regime (D=32, Y uniform(-2,2), gamma=0.5/D) at tail-tile sizes.
    X = randn(65, 32)
    Y = torch.rand(129, 32, generator=gen) * 4.0 - 2.0
    G = randn(65, 129)
    _save("c3like_n65_m129_d32", X, Y, G, 0.5 / 32, *_run(reference, X, Y, 0.5 / 32, G),
          "c3 distributions, tail tiles")

    # 4) The c4 regime (D=256, inputs N(0,1)/sqrt(2), gamma=1/D).
    X, Y = randn(16, 256) / 2 ** 0.5, randn(24, 256) / 2 ** 0.5
    G = randn(16, 24)
    _save("c4like_n16_m24_d256", X, Y, G, 1 / 256, *_run(reference, X, Y, 1 / 256, G),
          "c4 distributions")

    # 5) Exact duplicates (distance 0 -> K = 1) and near duplicates (cancellation).
    X = randn(40, 64)
    Y = torch.cat([X[:20].clone(), X[20:].clone() + 1e-3 * randn(20, 64), randn(9, 64)])
    G = randn(40, 49)
    _save("duplicates_n40_m49_d64", X, Y, G, 1 / 64, *_run(reference, X, Y, 1 / 64, G),
          "rows of Y equal / within 1e-3 of rows of X")

    # 6) Degenerate sizes: single element, D=1, and an empty X.
    X, Y = randn(1, 1), randn(1, 1)
    G = randn(1, 1)
    _save("single_n1_m1_d1", X, Y, G, 0.5, *_run(reference, X, Y, 0.5, G), "1x1, D=1")
    X, Y = randn(0, 3), randn(5, 3)
    G = randn(0, 5)
    _save("empty_n0_m5_d3", X, Y, G, 0.5, *_run(reference, X, Y, 0.5, G), "N=0")

    # 7) Large gamma: most of K underflows to 0, some entries subnormal.
    X, Y = randn(33, 16), randn(31, 16)
    G = randn(33, 31)
    _save("saturated_n33_m31_d16", X, Y, G, 4.0, *_run(reference, X, Y, 4.0, G),
          "gamma=4, K mostly 0")


if __name__ == "__main__":
    main()
