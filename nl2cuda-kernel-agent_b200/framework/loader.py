"""sm_100a loader (reference ``framework/loader.py:39-74``, ``load_kernel``).

The reference JIT-compiles each ``.cu`` into a pybind torch extension for ``CUDA_ARCHS``
(default "75,80").  Here the kernels are a C-ABI shared library built in-tree for sm_100a only:
``load_kernel`` (same signature) rebuilds ``lib/lib<name>.so`` with nvcc when a source is newer
than the library and returns it as a ``ctypes.CDLL``.  ``CUDA_ARCHS`` is accepted for
compatibility and must name 100a.  No fast-math (reference loader.py:6-9): the kernels use
IEEE fp32 arithmetic; the forward's exp is the documented ex2-based evaluation.

There is no CPU fallback: unlike the reference (loader.py:50-51) a missing GPU does not stop
the build, but calling into the library without an sm_100 device returns an error status,
which the Python layer raises as RuntimeError.
"""
import ctypes
import os
import shutil
import sys
import threading

_PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

import build as _build  # noqa: E402  (nl2cuda-kernel-agent_b200/build.py)

_ARCHS = [a.strip() for a in os.environ.get("CUDA_ARCHS", "100a").split(",") if a.strip()]
_lock = threading.Lock()
_loaded = {}


def _check_arch():
    if _ARCHS != ["100a"]:
        raise RuntimeError(f"CUDA_ARCHS={','.join(_ARCHS)!r}: this library is built for sm_100a "
                           "(B200) only; set CUDA_ARCHS=100a or leave it unset")


def load_kernel(name, sources=None, base_dir=None, extra_cuda_cflags=None, extra_cflags=None,
                verbose=False):
    """Build (if stale) and load lib/lib<name>.so; returns the ctypes.CDLL.

    ``sources`` are .cu files (absolute, or relative to ``base_dir``; default: all of csrc/).
    ``extra_cflags`` is accepted for signature compatibility (no host-only sources here).
    """
    del extra_cflags
    _check_arch()
    srcs = None
    if sources is not None:
        base = base_dir if base_dir is not None else _build.CSRC
        srcs = [s if os.path.isabs(s) else os.path.join(base, s) for s in sources]
        for s in srcs:
            if not os.path.exists(s):
                raise FileNotFoundError(f"source not found: {s}")
    with _lock:
        if name in _loaded:
            return _loaded[name]
        path = _build.lib_path(name)
        if _build.stale(name, srcs):
            if shutil.which(_build.NVCC) is None and not os.path.exists(path):
                raise RuntimeError(f"{path} is missing and nvcc is not available to build it")
            if shutil.which(_build.NVCC) is not None:
                _build.build(verbose=verbose, name=name, srcs=srcs,
                             extra_cuda_cflags=extra_cuda_cflags)
        lib = ctypes.CDLL(path)
        _loaded[name] = lib
        return lib
