"""Generate the cosine-similarity golden fixtures (``cos_*.npz``) from the reference's own code.

Runs the reference project's ``cases/cosine_sim/reference.py`` (``reference_forward`` and
``make_inputs``) with torch on the CPU, plus torch autograd for the backward, as the reference's
``framework/verify.py`` does (upstream gradient drawn from
``torch.Generator().manual_seed(seed + 10000)``).  The reference is imported from the path given
by ``--reference`` (default: the environment variable RBF_REFERENCE_ROOT); it is only needed to
regenerate the fixtures, never to run the tests.

Usage:  python tests/golden/make_golden_cosine.py --reference <path-to-reference-checkout>
"""
import argparse
import importlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(root, n, m, d):
    os.environ["COS_N"], os.environ["COS_M"], os.environ["COS_D"] = str(n), str(m), str(d)
    if root not in sys.path:
        sys.path.insert(0, root)
    for mod in [k for k in list(sys.modules) if k == "cases" or k.startswith("cases.")
                or k == "framework" or k.startswith("framework.")]:
        del sys.modules[mod]
    return importlib.import_module("cases.cosine_sim.reference")


def _run(reference, A, B, eps, dS):
    Ar = A.clone().requires_grad_(True)
    Br = B.clone().requires_grad_(True)
    S = reference.reference_forward({"A": Ar, "B": Br}, {"eps": eps})
    S.backward(dS)
    return S.detach(), Ar.grad.detach(), Br.grad.detach()


def _save(name, A, B, dS, eps, S, dA, dB, note):
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, A=A.numpy(), B=B.numpy(), dS=dS.numpy(), eps=np.float64(eps),
                        S=S.numpy(), dA=dA.numpy(), dB=dB.numpy(), note=np.array(note))
    print(f"wrote {path}  A{tuple(A.shape)} B{tuple(B.shape)}  ({note})")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("RBF_REFERENCE_ROOT"))
    args = ap.parse_args()
    if not args.reference:
        raise SystemExit("pass --reference <reference checkout> or set RBF_REFERENCE_ROOT")
    eps = 1e-8

    # 1) The reference's input generator and verify.py's gradient stream, at sizes the CPU
    #    finishes quickly (the default shape is 2048 x 2048 x 64).
    for seed, (n, m, d) in [(0, (96, 80, 64)), (1, (64, 64, 64)), (2, (64, 64, 64))]:
        reference = _import_reference(args.reference, n, m, d)
        inp = reference.make_inputs(seed, torch.float32, "cpu")
        g = torch.Generator(device="cpu").manual_seed(seed + 10_000)
        dS = torch.randn(n, m, dtype=torch.float32, generator=g)
        _save(f"cos_makeinputs_seed{seed}_n{n}_m{m}", inp["A"], inp["B"], dS, eps,
              *_run(reference, inp["A"], inp["B"], eps, dS),
              f"reference make_inputs(seed={seed}) COS_N={n} COS_M={m}; dS seed {seed + 10000}")

    reference = _import_reference(args.reference, 64, 64, 64)
    gen = torch.Generator().manual_seed(4321)

    def randn(*s):
        return torch.randn(*s, generator=gen, dtype=torch.float32)

    # 2) Ragged shape, odd D, M not a multiple of 4.
    A, B, dS = randn(37, 5), randn(50, 5), randn(37, 50)
    _save("cos_ragged_n37_m50_d5", A, B, dS, eps, *_run(reference, A, B, eps, dS), "ragged odd D")
    A, B, dS = randn(45, 40), randn(33, 40), randn(45, 33)
    _save("cos_ragged_n45_m33_d40", A, B, dS, eps, *_run(reference, A, B, eps, dS),
          "M % 4 != 0")

    # 3) D > 64 (feature slices), with rows of very different scale.
    A = randn(24, 130) * torch.logspace(-3, 3, 24).unsqueeze(1)
    B, dS = randn(20, 130), randn(24, 20)
    _save("cos_wide_n24_m20_d130", A, B, dS, eps, *_run(reference, A, B, eps, dS),
          "D=130, row norms 1e-3..1e3")

    # 4) Parallel / antiparallel / orthogonal rows (S = +-1, 0) and a zero row.
    base = randn(8, 16)
    A = torch.cat([base, torch.zeros(1, 16)])
    B = torch.cat([2.5 * base[:4], -0.5 * base[4:], randn(3, 16)])
    dS = randn(9, 11)
    _save("cos_aligned_n9_m11_d16", A, B, dS, eps, *_run(reference, A, B, eps, dS),
          "parallel, antiparallel rows and a zero row of A")

    # 5) Degenerate sizes.
    A, B, dS = randn(1, 1), randn(1, 1), randn(1, 1)
    _save("cos_single_n1_m1_d1", A, B, dS, eps, *_run(reference, A, B, eps, dS), "1x1, D=1")
    A, B, dS = randn(0, 3), randn(5, 3), randn(0, 5)
    _save("cos_empty_n0_m5_d3", A, B, dS, eps, *_run(reference, A, B, eps, dS), "N=0")


if __name__ == "__main__":
    main()
