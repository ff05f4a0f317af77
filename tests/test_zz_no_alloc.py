"""The allocation-free forward, rbf_sm100_forward_noalloc, called through the C ABI.

It exists for callers that cannot allocate device memory (an application whose allocator owns
the device heap, a runtime that forbids cudaMalloc on its hot path, a plugin interface with no
workspace argument): its workspace is a fixed array inside the library.  The tests check its K
against rbf_sm100_forward's and against the CPU oracle on two calls in a row (different inputs,
so a stale workspace from the first call would show), that the calls allocate no device memory,
that an over-capacity size is refused with RBF_ERR_TOO_LARGE, and that a device-side wait that
runs out is reported through rbf_sm100_forward_noalloc_read_status.
This file sorts last so that a run stopping at its first failure has run every other test.
"""
import ctypes
import os

import numpy as np
import pytest
import torch

from gpu_util import TOL, assert_gate, to_dev
from oracle import oracle

pytestmark = pytest.mark.gpu

RBF_ERR_TOO_LARGE = 8


def _noalloc(L, X, Y, K, gamma):
    vp = ctypes.c_void_p
    f = L.rbf_sm100_forward_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [vp, vp, vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_float, vp]
    s = torch.cuda.current_stream().cuda_stream
    return f(vp(X.data_ptr()), vp(Y.data_ptr()), vp(K.data_ptr()), X.shape[0], Y.shape[0],
             X.shape[1], ctypes.c_float(gamma), vp(s))


def test_noalloc_forward_matches_workspace_forward_twice(cuda_device):
    from cases.rbf import native
    L = native.lib()
    for call, (N, M, D, gamma, seed) in enumerate([(1000, 1028, 64, 1 / 64, 11),
                                                   (513, 260, 100, 0.01, 12)]):
        r = np.random.default_rng(seed)
        X, Y = to_dev(r.standard_normal((N, D)), r.standard_normal((M, D)))
        K = torch.full((N, M), float("nan"), device=cuda_device)
        st = _noalloc(L, X, Y, K, gamma)
        assert st == 0, (call, L.rbf_sm100_last_error_detail())
        torch.cuda.synchronize()
        ref = native.rbf_forward(X, Y, gamma)
        assert_gate(f"call {call} K", K.cpu().numpy(), ref.cpu().numpy(), TOL)
        rows = np.unique(r.integers(0, N, 16))
        assert_gate(f"call {call} K vs oracle", K.cpu().numpy()[rows],
                    oracle.forward_rows(X.cpu().numpy(), Y.cpu().numpy(), gamma, rows), TOL)


def test_noalloc_forward_allocates_no_device_memory(cuda_device):
    from cases.rbf import native
    L = native.lib()
    N = M = 4096  # the largest c1-sized call: (N + M) * 129 * 4 B, within the 16 MiB array
    gen = torch.Generator(device=cuda_device).manual_seed(5)
    X = torch.randn(N, 64, device=cuda_device, generator=gen)
    Y = torch.randn(M, 64, device=cuda_device, generator=gen)
    K = torch.empty(N, M, device=cuda_device)
    assert _noalloc(L, X, Y, K, 1 / 64) == 0  # warm-up: symbol lookup, module load
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    alloc0 = torch.cuda.memory_allocated()
    for _ in range(5):
        assert _noalloc(L, X, Y, K, 1 / 64) == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert torch.cuda.memory_allocated() == alloc0


def test_noalloc_wait_timeout_is_reported(cuda_device):
    from cases.rbf import native
    L = native.lib()
    rs = L.rbf_sm100_forward_noalloc_read_status
    rs.restype = ctypes.c_int
    rs.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]
    r = np.random.default_rng(3)
    X, Y = to_dev(r.standard_normal((256, 64)), r.standard_normal((300, 64)))
    K = torch.zeros(256, 300, device=cuda_device)
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    os.environ["RBF_DEBUG_SKIP_FIRST_LOAD"] = "1"
    os.environ["RBF_WAIT_TIMEOUT_MS"] = "100"
    try:
        assert _noalloc(L, X, Y, K, 1 / 64) == 0
        out = ctypes.c_int(-1)
        assert rs(s, ctypes.byref(out)) == 0
    finally:
        del os.environ["RBF_DEBUG_SKIP_FIRST_LOAD"]
        del os.environ["RBF_WAIT_TIMEOUT_MS"]
    assert out.value == 7  # RBF_ERR_TIMEOUT
    # A normal call right after is correct and reports OK.
    assert _noalloc(L, X, Y, K, 1 / 64) == 0
    out = ctypes.c_int(-1)
    assert rs(s, ctypes.byref(out)) == 0 and out.value == 0
    assert_gate("K after timeout", K.cpu().numpy(),
                oracle.forward(X.cpu().numpy(), Y.cpu().numpy(), 1 / 64), TOL)


def test_noalloc_rejects_sizes_beyond_capacity(cuda_device):
    from cases.rbf import native
    L = native.lib()
    L.rbf_sm100_forward_noalloc_capacity.restype = ctypes.c_size_t
    cap = L.rbf_sm100_forward_noalloc_capacity()
    assert cap == 16 << 20
    X = torch.zeros(40000, 64, device=cuda_device)  # (40000 + 40000) * 129 * 4 B > 16 MiB
    K = torch.zeros(1, 1, device=cuda_device)
    vp = ctypes.c_void_p
    f = L.rbf_sm100_forward_noalloc
    f.argtypes = [vp, vp, vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_float, vp]
    st = f(vp(X.data_ptr()), vp(X.data_ptr()), vp(K.data_ptr()), 40000, 40000, 64,
           ctypes.c_float(0.1), vp(0))
    assert st == RBF_ERR_TOO_LARGE
    assert b"scratch" in L.rbf_sm100_last_error_detail()
