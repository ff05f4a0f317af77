"""Build the sm_100a shared library of this package: lib/librbf_sm100.so.

One nvcc invocation per .cu (objects cached by mtime under _build/), then a single
``nvcc -shared`` link.  The library exports only the C ABI of include/rbf_sm100.h.  Used by
__graft_entry__.build(), by framework/loader.py (rebuild when a source is newer than the .so)
and directly:  python nl2cuda-kernel-agent_b200/build.py [--verbose] [--ptxas-info]
"""
import argparse
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
INCLUDE = os.path.join(ROOT, "include")

NVCC = os.environ.get("NVCC", "nvcc")
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler",
          "-fvisibility=hidden", "-I", INCLUDE, "-I", CSRC]


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def lib_path(name="rbf_sm100"):
    return os.path.join(PKG, "lib", f"lib{name}.so")


def headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h")))


def _newest(paths):
    return max((os.path.getmtime(p) for p in paths), default=0.0)


def stale(name="rbf_sm100", srcs=None):
    lib = lib_path(name)
    if not os.path.exists(lib):
        return True
    srcs = sources() if srcs is None else list(srcs)
    return _newest(srcs + headers() + [__file__]) > os.path.getmtime(lib)


def build(verbose=False, ptxas_info=False, force=False, name="rbf_sm100", srcs=None,
          extra_cuda_cflags=None):
    """Compile `srcs` (default: every csrc/*.cu) for sm_100a and link lib/lib<name>.so."""
    lib = lib_path(name)
    obj_dir = os.path.join(BUILD, name)
    os.makedirs(obj_dir, exist_ok=True)
    os.makedirs(os.path.dirname(lib), exist_ok=True)
    hdr_time = max(_newest(headers()), os.path.getmtime(__file__))
    extra = list(extra_cuda_cflags or [])
    objs = []
    for src in (sources() if srcs is None else list(srcs)):
        obj = os.path.join(obj_dir, os.path.basename(src).rsplit(".", 1)[0] + ".o")
        objs.append(obj)
        if (not force and os.path.exists(obj) and not ptxas_info
                and os.path.getmtime(obj) >= max(os.path.getmtime(src), hdr_time)):
            continue
        cmd = [NVCC, *ARCH_FLAGS, *COMMON, *extra, "-c", src, "-o", obj]
        if ptxas_info:
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    cmd = [NVCC, *ARCH_FLAGS, "-shared", "-o", lib + ".tmp", *objs]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(lib + ".tmp", lib)
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, ptxas_info=a.ptxas_info, force=a.force))
    sys.exit(0)
