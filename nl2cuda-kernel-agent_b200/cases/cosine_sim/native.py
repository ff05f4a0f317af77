"""ctypes binding of the cosine-similarity C ABI (include/cos_sm100.h) for torch tensors.

``cos_forward(A, B, eps) -> S`` and ``cos_backward(...) -> [dA, dB]`` replace the reference's
torch-extension calls (reference ``cases/cosine_sim/kernels/cosine_sim.cu:104-125``), with the
same argument meaning.  The state the reference passes from forward to backward (Ah, Bh, invA,
invB) is the workspace here.  Kernels run on torch's current CUDA stream; errors are raised as
RuntimeError; there is no fallback -- a missing library or a non-sm_100 device raises.
"""
import ctypes
import threading

import torch

from cases.rbf import native as _rbf

_lock = threading.Lock()
_bound = None

_F = ctypes.c_void_p
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t


def lib():
    """The library (shared with the RBF case) with the cos_sm100_* signatures declared."""
    global _bound
    with _lock:
        if _bound is None:
            L = _rbf.lib()
            for fn in ("cos_sm100_forward_workspace_bytes", "cos_sm100_backward_workspace_bytes"):
                getattr(L, fn).restype = _SZ
                getattr(L, fn).argtypes = [_I64, _I64, _I64]
            L.cos_sm100_forward.restype = ctypes.c_int
            L.cos_sm100_forward.argtypes = [_F, _F, _F, _I64, _I64, _I64, ctypes.c_float, _F, _SZ,
                                            _F]
            L.cos_sm100_backward_prepared.restype = ctypes.c_int
            L.cos_sm100_backward_prepared.argtypes = [_F, _F, _F, _I64, _I64, _I64,
                                                      ctypes.c_float, _F, _SZ, _F]
            L.cos_sm100_backward.restype = ctypes.c_int
            L.cos_sm100_backward.argtypes = [_F, _F, _F, _F, _F, _I64, _I64, _I64, ctypes.c_float,
                                             _F, _SZ, _F]
            _bound = L
    return _bound


def workspace_bytes(N, M, D):
    """Bytes of a workspace valid for both the forward and the prepared backward."""
    L = lib()
    return max(L.cos_sm100_forward_workspace_bytes(N, M, D),
               L.cos_sm100_backward_workspace_bytes(N, M, D), 16)


def _shapes(A, B):
    _rbf.check_2d(("A", "B"), (A, B))
    if A.size(1) != B.size(1):
        raise RuntimeError("A, B must share feature dim D")
    if A.device != B.device:
        raise RuntimeError("A, B must be on the same device")


def forward_with_workspace(A, B, eps):
    """S and the filled workspace (normalised rows and norms, reused by the backward)."""
    _shapes(A, B)
    A, B = _rbf.operand(A), _rbf.operand(B)
    N, D = A.shape
    M = B.size(0)
    with torch.cuda.device(A.device):
        S = torch.empty((N, M), dtype=torch.float32, device=A.device)
        ws = torch.empty(workspace_bytes(N, M, D), dtype=torch.uint8, device=A.device)
        _rbf.check(lib().cos_sm100_forward(_rbf.ptr(A), _rbf.ptr(B), _rbf.ptr(S), N, M, D,
                                           float(eps), _rbf.ptr(ws), ws.numel(),
                                           _rbf.stream_of(A.device)), "cos_sm100_forward")
    return S, ws


def cos_forward(A, B, eps):
    """S[i,j] = A[i].B[j] / ((|A[i]| + eps)(|B[j]| + eps)) for A [N,D], B [M,D] (fp32, CUDA)."""
    return forward_with_workspace(A, B, eps)[0]


def cos_backward(dS, N, M, D, eps, workspace=None, A=None, B=None):
    """[dA, dB] of sum(dS * S).  ``workspace`` from ``forward_with_workspace`` of the same A, B
    (``cos_sm100_backward_prepared``), or else A and B (``cos_sm100_backward``)."""
    _rbf.check_2d(("dS",), (dS,))
    if tuple(dS.shape) != (N, M):
        raise RuntimeError("shape mismatch: dS must be [N, M]")
    dS = _rbf.operand(dS)
    dev = dS.device
    with torch.cuda.device(dev):
        dA = torch.empty((N, D), dtype=torch.float32, device=dev)
        dB = torch.empty((M, D), dtype=torch.float32, device=dev)
        if workspace is not None:
            _rbf.check(lib().cos_sm100_backward_prepared(
                _rbf.ptr(dS), _rbf.ptr(dA), _rbf.ptr(dB), N, M, D, float(eps),
                _rbf.ptr(workspace), workspace.numel(), _rbf.stream_of(dev)),
                "cos_sm100_backward_prepared")
        else:
            if A is None or B is None:
                raise RuntimeError("cos_backward needs the forward's workspace, or A and B")
            _shapes(A, B)
            A, B = _rbf.operand(A), _rbf.operand(B)
            ws = torch.empty(workspace_bytes(N, M, D), dtype=torch.uint8, device=dev)
            _rbf.check(lib().cos_sm100_backward(
                _rbf.ptr(A), _rbf.ptr(B), _rbf.ptr(dS), _rbf.ptr(dA), _rbf.ptr(dB), N, M, D,
                float(eps), _rbf.ptr(ws), ws.numel(), _rbf.stream_of(dev)), "cos_sm100_backward")
    return [dA, dB]
