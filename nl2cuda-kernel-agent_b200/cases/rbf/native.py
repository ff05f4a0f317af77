"""ctypes binding of the sm_100a C ABI (include/rbf_sm100.h) for torch tensors.

``rbf_forward(X, Y, gamma) -> K`` and ``rbf_backward(X, Y, G, K, gamma) -> [dX, dY]`` are the
calls of the reference's torch extensions (reference ``cases/rbf/kernels/rbf_forward.cu:94-116``
and ``rbf_backward.cu:59-84``) with the same argument checks, raised as RuntimeError as
TORCH_CHECK does.  Differences: kernels run on torch's current CUDA stream (the reference uses
the legacy default stream), every CUDA error is reported, and outputs / workspace come from
torch's caching allocator.

There is no fallback: if the library is missing or the device is not sm_100, the call raises.
"""
import ctypes
import threading

import torch

from framework.loader import load_kernel

_lock = threading.Lock()
_lib = None

_F = ctypes.c_void_p
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t


def lib():
    """The loaded C-ABI library (built on first use when a source is newer than the .so)."""
    global _lib
    with _lock:
        if _lib is None:
            L = load_kernel("rbf_sm100")
            L.rbf_sm100_strerror.restype = ctypes.c_char_p
            L.rbf_sm100_strerror.argtypes = [ctypes.c_int]
            L.rbf_sm100_last_error_detail.restype = ctypes.c_char_p
            L.rbf_sm100_last_error_detail.argtypes = []
            L.rbf_sm100_version.restype = ctypes.c_int
            L.rbf_sm100_launch_count.restype = ctypes.c_uint64
            L.rbf_sm100_launch_count.argtypes = []
            for fn in ("rbf_sm100_forward_workspace_bytes", "rbf_sm100_backward_workspace_bytes"):
                getattr(L, fn).restype = _SZ
                getattr(L, fn).argtypes = [_I64, _I64, _I64]
            L.rbf_sm100_forward.restype = ctypes.c_int
            L.rbf_sm100_forward.argtypes = [_F, _F, _F, _I64, _I64, _I64, ctypes.c_float, _F,
                                            _SZ, _F]
            for fn in ("rbf_sm100_backward", "rbf_sm100_backward_prepared",
                       "rbf_sm100_backward_shard", "rbf_sm100_forward_backward"):
                getattr(L, fn).restype = ctypes.c_int
                getattr(L, fn).argtypes = [_F, _F, _F, _F, _F, _F, _I64, _I64, _I64,
                                           ctypes.c_float, _F, _SZ, _F]
            L.rbf_sm100_backward_shard_routed.restype = ctypes.c_int
            L.rbf_sm100_backward_shard_routed.argtypes = [
                _F, _F, _F, _F, _F, _I64, _I64, _I64, ctypes.c_float, _F, _SZ,
                ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, ctypes.c_int, _F, _F]
            L.rbf_sm100_dy_exchange.restype = ctypes.c_int
            L.rbf_sm100_dy_exchange.argtypes = [
                _F, _I64, _I64, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p),
                ctypes.c_int, ctypes.c_int, _F, _F, _F, _SZ, _F]
            L.rbf_sm100_read_status.restype = ctypes.c_int
            L.rbf_sm100_read_status.argtypes = [_F, _F, ctypes.POINTER(ctypes.c_int)]
            _lib = L
    return _lib


def check(status, what):
    """Raise RuntimeError for a non-zero rbf_status."""
    if status != 0:
        L = lib()
        raise RuntimeError(f"{what}: {L.rbf_sm100_strerror(status).decode()} "
                           f"({L.rbf_sm100_last_error_detail().decode()})")


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t.numel() else ctypes.c_void_p(0)


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _operand(t):
    """Contiguous and 16-byte aligned (the ABI's pointer rule); copies only if needed."""
    t = t.contiguous()
    if t.numel() and t.data_ptr() % 16:
        t = t.clone()
    return t


def _check_2d(names, tensors):
    if not all(t.is_cuda for t in tensors):
        raise RuntimeError(f"{', '.join(names)} must be CUDA tensors")
    if not all(t.dtype == torch.float32 for t in tensors):
        raise RuntimeError(f"{', '.join(names)} must be float32")
    if not all(t.dim() == 2 for t in tensors):
        raise RuntimeError(f"{', '.join(names)} must be 2D")


def workspace_bytes(N, M, D):
    """Bytes of a workspace valid for both the forward and the prepared backward."""
    L = lib()
    return max(L.rbf_sm100_forward_workspace_bytes(N, M, D),
               L.rbf_sm100_backward_workspace_bytes(N, M, D))


def new_workspace(N, M, D, device):
    return torch.empty(max(workspace_bytes(N, M, D), 16), dtype=torch.uint8, device=device)


def forward_with_workspace(X, Y, gamma):
    """K and the filled workspace (the prepared X/Y split the backward can reuse)."""
    _check_2d(("X", "Y"), (X, Y))
    if X.size(1) != Y.size(1):
        raise RuntimeError("X, Y must share feature dim D")
    if X.device != Y.device:
        raise RuntimeError("X, Y must be on the same device")
    X, Y = _operand(X), _operand(Y)
    N, D = X.shape
    M = Y.size(0)
    with torch.cuda.device(X.device):
        K = torch.empty((N, M), dtype=torch.float32, device=X.device)
        ws = new_workspace(N, M, D, X.device)
        check(lib().rbf_sm100_forward(_ptr(X), _ptr(Y), _ptr(K), N, M, D, float(gamma),
                                      _ptr(ws), ws.numel(), _stream(X.device)),
              "rbf_sm100_forward")
    return K, ws


def rbf_forward(X, Y, gamma):
    """K = exp(-gamma * ||x_i - y_j||^2) for X [N,D], Y [M,D] (fp32 CUDA tensors)."""
    return forward_with_workspace(X, Y, gamma)[0]


def rbf_backward(X, Y, G, K, gamma, workspace=None, entry="rbf_sm100_backward"):
    """[dX, dY] of sum(G * K).  ``workspace`` from ``forward_with_workspace`` of the same X, Y
    skips the split pass (``rbf_sm100_backward_prepared``)."""
    _check_2d(("X", "Y", "G", "K"), (X, Y, G, K))
    X, Y, G, K = _operand(X), _operand(Y), _operand(G), _operand(K)
    N, D = X.shape
    M = Y.size(0)
    if Y.size(1) != D or tuple(G.shape) != (N, M) or tuple(K.shape) != (N, M):
        raise RuntimeError("shape mismatch: need X [N,D], Y [M,D], G and K [N,M]")
    with torch.cuda.device(X.device):
        dX = torch.empty_like(X)
        dY = torch.empty_like(Y)
        if workspace is not None:
            fn, ws = lib().rbf_sm100_backward_prepared, workspace
        else:
            fn, ws = getattr(lib(), entry), new_workspace(N, M, D, X.device)
        check(fn(_ptr(X), _ptr(Y), _ptr(G), _ptr(K), _ptr(dX), _ptr(dY), N, M, D, float(gamma),
                 _ptr(ws), ws.numel(), _stream(X.device)), fn.__name__)
    return [dX, dY]


def rbf_forward_backward(X, Y, G, gamma, return_workspace=False):
    """[K, dX, dY] in one call (``rbf_sm100_forward_backward``): the forward of X, Y and the
    backward of sum(G * K), for a G known before the forward; the same values as
    ``forward_with_workspace`` followed by ``rbf_backward`` with that workspace.  With
    ``return_workspace`` the workspace (its status word: ``read_status``) is appended."""
    _check_2d(("X", "Y", "G"), (X, Y, G))
    X, Y, G = _operand(X), _operand(Y), _operand(G)
    N, D = X.shape
    M = Y.size(0)
    if Y.size(1) != D or tuple(G.shape) != (N, M):
        raise RuntimeError("shape mismatch: need X [N,D], Y [M,D], G [N,M]")
    with torch.cuda.device(X.device):
        K = torch.empty((N, M), dtype=torch.float32, device=X.device)
        dX = torch.empty_like(X)
        dY = torch.empty_like(Y)
        ws = new_workspace(N, M, D, X.device)
        check(lib().rbf_sm100_forward_backward(_ptr(X), _ptr(Y), _ptr(G), _ptr(K), _ptr(dX),
                                               _ptr(dY), N, M, D, float(gamma), _ptr(ws),
                                               ws.numel(), _stream(X.device)),
              "rbf_sm100_forward_backward")
    return [K, dX, dY, ws] if return_workspace else [K, dX, dY]


# The ctypes helpers above, shared with the other case bound to this library (cosine_sim).
check_2d = _check_2d
operand = _operand
ptr = _ptr
stream_of = _stream


def launch_count():
    """Kernels this library has enqueued in this process."""
    return int(lib().rbf_sm100_launch_count())


def read_status(workspace):
    """Device status word of ``workspace`` (0 = ok, 7 = a bounded device wait timed out)."""
    out = ctypes.c_int(0)
    check(lib().rbf_sm100_read_status(_ptr(workspace), _stream(workspace.device),
                                      ctypes.byref(out)), "rbf_sm100_read_status")
    return out.value


def rbf_backward_shard_routed(X, Y, G, K, gamma, workspace, route):
    """dX of this rank's rows; the dY partial is accumulated into this rank's slot of ``route``
    (a ``shard.RoutedDy``) instead of being returned.  ``workspace`` from
    ``forward_with_workspace`` of the same X, Y.  Complete the step with ``dy_exchange``."""
    _check_2d(("X", "Y", "G", "K"), (X, Y, G, K))
    X, Y, G, K = _operand(X), _operand(Y), _operand(G), _operand(K)
    N, D = X.shape
    M = Y.size(0)
    if Y.size(1) != D or tuple(G.shape) != (N, M) or tuple(K.shape) != (N, M):
        raise RuntimeError("shape mismatch: need X [N,D], Y [M,D], G and K [N,M]")
    with torch.cuda.device(X.device):
        dX = torch.empty_like(X)
        check(lib().rbf_sm100_backward_shard_routed(
            _ptr(X), _ptr(Y), _ptr(G), _ptr(K), _ptr(dX), N, M, D, float(gamma), _ptr(workspace),
            workspace.numel(), route.dy_ptrs, route.world, route.rank, _ptr(route.counters),
            _stream(X.device)), "rbf_sm100_backward_shard_routed")
    return dX


def dy_exchange(route, workspace, out=None):
    """Barrier across ranks, then the full dY [M, D] gathered from the owners' slots."""
    dev = route.device
    with torch.cuda.device(dev):
        dY = out if out is not None else torch.empty((route.M, route.D), dtype=torch.float32,
                                                     device=dev)
        check(lib().rbf_sm100_dy_exchange(
            _ptr(dY), route.M, route.D, route.dy_ptrs, route.flag_ptrs, route.world, route.rank,
            _ptr(route.counters), route.counters.data_ptr() + 4, _ptr(workspace),
            workspace.numel(), _stream(dev)), "rbf_sm100_dy_exchange")
    return dY
