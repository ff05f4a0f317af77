"""Per-role timeline of CTA 0 of the tensor-core backward (development tool).

Builds the library with -DRBF_TRACE under its own name (lib/librbf_trace.so; the product library
is left alone), runs the RBF or the cosine-similarity backward a few times at one size, and
prints, for each role of CTA 0, its events as code@microseconds since the first event:

    python -m framework.timeline [--case rbf|cosine_sim] [--n 4096] [--dyn-pct 0]

Roles and codes (rbf_bwd_tc.cu):
    PROD  10+p   strip (or stage) p of a tile issued
    dY    10+h   W^T half h written by the C-warps;     20+s  X chunk s landed
    dX    20+s   W of strip s written and its Y rows landed
    C0    10     strip landed; 20+h  W^T half h free;   30+h  half h written;  40  strip released
    R0    10+s   strip s landed; 20+s W buffer free;    30+s  W written;       40  dX flushed
    C3 / R3      as C0 / R0 for the fourth quadrant
Run it from the package directory on one GPU.
"""
import argparse
import ctypes
import os
import sys

_PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

ROLES = ["PROD", "-", "dY", "dX", "C0", "R0", "C3", "R3"]


def load_trace_library():
    """Build lib/librbf_trace.so (-DRBF_TRACE) and make the bindings use it."""
    import build as _build
    import framework.loader as loader
    path = _build.build(name="rbf_trace", extra_cuda_cflags=["-DRBF_TRACE"])
    loader._loaded["rbf_sm100"] = ctypes.CDLL(path)
    return loader._loaded["rbf_sm100"]


def format_timeline(buf, counts, names=ROLES, max_events=120):
    """Lines 'ROLE code@us ...' from the packed (code << 56 | globaltimer ns) trace buffers."""
    mask = (1 << 56) - 1
    starts = [int(buf[r][0]) & mask for r in range(len(names)) if counts[r]]
    if not starts:
        return []
    t0 = min(starts)
    lines = []
    for r, name in enumerate(names):
        if not counts[r]:
            continue
        ev = [(int(x) >> 56, ((int(x) & mask) - t0) / 1000.0) for x in buf[r][:counts[r]]]
        lines.append(name + " " + " ".join(f"{c}@{t:.2f}" for c, t in ev[:max_events]))
    return lines


def format_spans(sp, ctas):
    """Summary lines of the per-CTA records of the last traced run (g_cta_span in
    rbf_bwd_tc.cu), in microseconds since the earliest CTA start: start (after set-up), release
    by the previous kernel, last strip issued, end; and the tiles each CTA ran."""
    import numpy as np
    m48 = (1 << 48) - 1
    sp = sp[:ctas].astype(np.int64)
    start, end, rel = sp[:, 0] & m48, sp[:, 1] & m48, sp[:, 2] & m48
    last, tiles = sp[:, 3] & m48, sp[:, 3] >> 48
    t0 = start.min()

    def q(name, v):
        v = (v - t0) / 1000.0
        return (f"{name:<11} min {v.min():7.2f}  p50 {np.median(v):7.2f}  "
                f"p90 {np.percentile(v, 90):7.2f}  max {v.max():7.2f}")
    lines = [q("start", start), q("released", rel), q("last strip", last), q("end", end)]
    dur = (end - rel) / 1000.0
    tail = (end - last) / 1000.0
    lines.append(f"release->end  min {dur.min():7.2f}  p50 {np.median(dur):7.2f}  max {dur.max():7.2f}")
    lines.append(f"last strip->end  p50 {np.median(tail):.2f}  max {tail.max():.2f}")
    vals, counts = np.unique(tiles, return_counts=True)
    lines.append("tiles per CTA: " + ", ".join(f"{int(v)} x{int(c)}" for v, c in zip(vals, counts)))
    for v in vals:
        sel = tiles == v
        lines.append(f"  {int(v)} tiles: end p50 {np.median((end[sel] - t0) / 1000.0):.2f}  "
                     f"release->end p50 {np.median(dur[sel]):.2f}")
    return lines


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--case", choices=("rbf", "cosine_sim"), default="rbf")
    ap.add_argument("--n", type=int, default=4096, help="N = M (D = 64)")
    ap.add_argument("--dyn-pct", default="0", help="RBF_BWD_DYN_PCT for the traced runs")
    ap.add_argument("--spans", action="store_true",
                    help="also summarise every CTA's start, release, last strip issue and end")
    args = ap.parse_args(argv)
    import numpy as np
    import torch
    L = load_trace_library()
    from cases.cosine_sim import native as cn
    from cases.rbf import native
    os.environ["RBF_BWD_DYN_PCT"] = args.dyn_pct
    N = M = args.n
    D = 64
    X = torch.randn(N, D, device="cuda")
    Y = torch.randn(M, D, device="cuda")
    G = torch.randn(N, M, device="cuda")
    if args.case == "rbf":
        K, ws = native.forward_with_workspace(X, Y, 1 / D)
        run = lambda: native.rbf_backward(X, Y, G, K, 1 / D, workspace=ws)  # noqa: E731
    else:
        _, ws = cn.forward_with_workspace(X, Y, 1e-8)
        run = lambda: cn.cos_backward(G, N, M, D, 1e-8, workspace=ws)  # noqa: E731
    buf = np.zeros((8, 1024), np.uint64)
    n = np.zeros(8, np.int32)
    for _ in range(3):  # the last run's trace is kept (the first ones warm up)
        run()
        torch.cuda.synchronize()
        L.rbf_debug_trace(buf.ctypes.data_as(ctypes.c_void_p), n.ctypes.data_as(ctypes.c_void_p))
    print(f"CTA 0 timeline, {args.case} backward, N = M = {N}, D = {D} (microseconds)")
    print("\n".join(format_timeline(buf, n)))
    if args.spans:
        sp = np.zeros((1024, 4), np.uint64)
        L.rbf_debug_spans(sp.ctypes.data_as(ctypes.c_void_p))
        sms = torch.cuda.get_device_properties(0).multi_processor_count
        print("\n".join(format_spans(sp, min(sms, N // 128 * (M // 128)))))
    return 0


if __name__ == "__main__":
    sys.exit(main())
