"""The C-ABI library loads, exports every symbol include/*.h declares (rbf_sm100.h and
cos_sm100.h), and rejects bad arguments on the host (no GPU needed; no compute call is made)."""
import ctypes
import glob
import os
import re

import pytest

from conftest import has_gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = sorted(glob.glob(os.path.join(ROOT, "include", "*.h")))

RBF_OK, INVALID, MISALIGNED, WORKSPACE, UNSUPPORTED, CUDA, NO_DEVICE = 0, 1, 2, 3, 4, 5, 6


def declared_functions():
    text = "".join(open(h).read() for h in HEADERS)
    return sorted(set(re.findall(r"RBF_API\s+[\w\s\*]+?\b((?:rbf|cos)_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from cases.rbf import native
    return native.lib()


def test_header_declares_the_boundary():
    fns = declared_functions()
    for f in ("rbf_sm100_forward", "rbf_sm100_backward", "rbf_sm100_forward_workspace_bytes",
              "rbf_sm100_backward_workspace_bytes", "rbf_sm100_strerror", "rbf_forward_cuda",
              "rbf_backward_cuda", "cos_sm100_forward", "cos_sm100_backward",
              "cos_sm100_backward_prepared", "cos_sm100_forward_workspace_bytes",
              "cos_sm100_backward_workspace_bytes"):
        assert f in fns


def test_library_exports_every_declared_symbol(lib):
    missing = [f for f in declared_functions() if not hasattr(lib, f)]
    assert not missing, missing


def test_strerror_covers_all_codes(lib):
    for code in range(0, 9):
        assert lib.rbf_sm100_strerror(code)
    assert b"unknown" in lib.rbf_sm100_strerror(99)


def test_workspace_sizes(lib):
    f = lib.rbf_sm100_forward_workspace_bytes
    b = lib.rbf_sm100_backward_workspace_bytes
    assert f(-1, 1, 1) == 0
    assert f(4096, 4096, 64) >= 2 * 2 * 4096 * 64 * 4 + 2 * 4096 * 4
    assert b(4096, 4096, 64) >= f(4096, 4096, 64)
    assert f(100, 100, 33) > f(100, 100, 32)  # D padded to the next multiple of 32


def _fwd(lib, X, Y, K, N, M, D, gamma, ws, wsb):
    vp = ctypes.c_void_p
    return lib.rbf_sm100_forward(vp(X), vp(Y), vp(K), N, M, D, ctypes.c_float(gamma), vp(ws),
                                 wsb, vp(0))


def test_host_side_validation(lib):
    A = 1 << 20  # fake 16-byte aligned addresses: validation fails before they are touched
    wsb = lib.rbf_sm100_forward_workspace_bytes(8, 8, 4)
    assert _fwd(lib, A, A, A, -1, 8, 4, 0.5, A, wsb) == INVALID
    assert _fwd(lib, A, A, A, 8, 8, 5000, 0.5, A, 1 << 30) == UNSUPPORTED
    assert _fwd(lib, A, A, A, 8, 8, 4, float("nan"), A, wsb) == INVALID
    assert _fwd(lib, A + 4, A, A, 8, 8, 4, 0.5, A, wsb) == MISALIGNED
    assert _fwd(lib, 0, A, A, 8, 8, 4, 0.5, A, wsb) == INVALID
    assert _fwd(lib, A, A, A, 8, 8, 4, 0.5, A, wsb - 1) == WORKSPACE
    assert _fwd(lib, A, A, A, 8, 8, 4, 0.5, 0, wsb) == WORKSPACE
    assert b"workspace" in lib.rbf_sm100_last_error_detail()


@pytest.mark.skipif(has_gpu(), reason="checks the no-device path")
def test_valid_call_without_device_fails_loudly(lib):
    A = 1 << 20
    wsb = lib.rbf_sm100_forward_workspace_bytes(8, 8, 4)
    assert _fwd(lib, A, A, A, 8, 8, 4, 0.5, A, wsb) == NO_DEVICE


def test_native_refuses_cpu_tensors():
    import torch
    from cases.rbf import native, op
    X = torch.randn(4, 3)
    with pytest.raises(RuntimeError, match="CUDA"):
        native.rbf_forward(X, X, 0.5)
    with pytest.raises(RuntimeError, match="CUDA"):
        op.candidate({"X": X, "Y": X}, {"gamma": 0.5})


def test_cosine_host_side_validation(lib):
    from cases.cosine_sim import native as cos_native
    L = cos_native.lib()
    vp = ctypes.c_void_p
    A = 1 << 20
    wsb = L.cos_sm100_backward_workspace_bytes(8, 8, 4)
    assert wsb >= L.cos_sm100_forward_workspace_bytes(8, 8, 4) > 0

    def fwd(a, b, s, N, M, D, eps, ws, n):
        return L.cos_sm100_forward(vp(a), vp(b), vp(s), N, M, D, ctypes.c_float(eps), vp(ws), n,
                                   vp(0))

    def bwd(ds, da, db, N, M, D, eps, ws, n):
        return L.cos_sm100_backward_prepared(vp(ds), vp(da), vp(db), N, M, D,
                                             ctypes.c_float(eps), vp(ws), n, vp(0))

    assert fwd(A, A, A, 8, -1, 4, 1e-8, A, wsb) == INVALID
    assert fwd(A, A, A, 8, 8, 4, float("inf"), A, wsb) == INVALID
    assert b"eps" in lib.rbf_sm100_last_error_detail()
    assert fwd(A, A + 8, A, 8, 8, 4, 1e-8, A, wsb) == MISALIGNED
    assert fwd(A, A, A, 8, 8, 4, 1e-8, A, 16) == WORKSPACE
    assert bwd(A, A, A, 8, 8, 4, 1e-8, A, wsb - 1) == WORKSPACE
    assert bwd(0, A, A, 8, 8, 4, 1e-8, A, wsb) == INVALID
    assert bwd(A, A, A, 8, 8, 5000, 1e-8, A, 1 << 30) == UNSUPPORTED


def test_deterministic_backward_workspace_holds_the_tile_slots(lib, monkeypatch):
    """RBF_DETERMINISTIC=1 (read at every call) adds the per-tile partial slots of dX and dY,
    4 * (tiles_j * Npad + tiles_i * M) * (D + 1) bytes, to the backward workspace."""
    b = lib.rbf_sm100_backward_workspace_bytes
    N, M, D = 300, 400, 64
    monkeypatch.delenv("RBF_DETERMINISTIC", raising=False)
    base = b(N, M, D)
    monkeypatch.setenv("RBF_DETERMINISTIC", "1")
    det = b(N, M, D)
    tiles_j, tiles_i, npad = 4, 3, 384
    assert det - base >= 4 * (tiles_j * npad + tiles_i * M) * (D + 1)
    assert det - base <= 4 * (tiles_j * npad + tiles_i * M) * (D + 1) + 4 * 256
    ragged = b(N, 401, D)  # M % 4 != 0: the CUDA-core kernels, deterministic already
    monkeypatch.setenv("RBF_DETERMINISTIC", "0")
    assert b(N, M, D) == base
    assert b(N, 401, D) == ragged
