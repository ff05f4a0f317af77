"""Loading the golden fixtures of tests/golden, generated from the reference's own code: the RBF
fixtures by tests/golden/make_golden.py, the cosine-similarity ones (``cos_*``) by
tests/golden/make_golden_cosine.py."""
import glob
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _all():
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "*.npz")))


def names():
    """The RBF fixtures."""
    return [n for n in _all() if not n.startswith("cos_")]


def cos_names():
    """The cosine-similarity fixtures."""
    return [n for n in _all() if n.startswith("cos_")]


def load(name):
    with np.load(os.path.join(GOLDEN, name + ".npz")) as z:
        return {k: z[k] for k in z.files}
