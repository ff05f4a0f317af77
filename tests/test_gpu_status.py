"""Failure detection on the GPU without a GPU fault: a device-side wait that runs out.

RBF_DEBUG_SKIP_FIRST_LOAD=1 makes CTA 0 of the tensor-core kernels skip filling its first
pipeline stage, so the consumer's bounded mbarrier wait (RBF_WAIT_TIMEOUT_MS) expires.  The
kernel then records RBF_ERR_TIMEOUT in the workspace status word, drains its own copies in
flight, frees TMEM and returns; the context stays usable, which the test checks by running a
normal call right after.
"""
import os

import numpy as np
import pytest
import torch

from gpu_util import assert_gate, to_dev
from oracle import oracle

pytestmark = pytest.mark.gpu

RBF_ERR_TIMEOUT = 7


def test_forward_wait_timeout_is_reported_and_context_survives(cuda_device):
    from cases.rbf import native
    r = np.random.default_rng(0)
    X, Y = r.standard_normal((256, 64)), r.standard_normal((256, 64))
    Xd, Yd = to_dev(X, Y)
    os.environ["RBF_DEBUG_SKIP_FIRST_LOAD"] = "1"
    os.environ["RBF_WAIT_TIMEOUT_MS"] = "100"
    try:
        K, ws = native.forward_with_workspace(Xd, Yd, 1 / 64)
        status = native.read_status(ws)
    finally:
        del os.environ["RBF_DEBUG_SKIP_FIRST_LOAD"]
        del os.environ["RBF_WAIT_TIMEOUT_MS"]
    assert status == RBF_ERR_TIMEOUT
    # The context is intact: a normal call right after is correct and reports no error.
    K, ws = native.forward_with_workspace(Xd, Yd, 1 / 64)
    assert native.read_status(ws) == 0
    assert_gate("K", K.cpu().numpy(), oracle.forward(X.astype(np.float32), Y.astype(np.float32), 1 / 64))
