"""Speed gate against ``torch.compile(case.reference_forward)`` (reference
``framework/bench.py:31-178``).

Forward and backward are timed separately with CUDA events, a synchronize on both sides of
every timed call.  Each repeat reports the geometric mean of ``iters`` timings; a measurement
whose coefficient of variation across repeats exceeds the protocol threshold is retaken (at most
``max_retries`` times) and the lowest-CV attempt is kept.  The backward graph is rebuilt outside
the timed region, so only ``out.backward(G)`` is timed.  G is seeded with 777 (reference
bench.py:141).  The candidate passes at >= ``speedup_target`` on both passes with every CV in
bounds.
"""
import math
import statistics

import torch

from framework.protocol import PROTOCOL, dtype_of


def _geomean(xs):
    return math.exp(sum(math.log(x) for x in xs) / len(xs))


def _time_call(fn):
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b)


def _timings(fn, warmup, iters):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    return [_time_call(fn) for _ in range(iters)]


def _backward_timings(make_bwd, warmup, iters):
    for _ in range(warmup):
        make_bwd()()
    torch.cuda.synchronize()
    out = []
    for _ in range(iters):
        bwd = make_bwd()
        out.append(_time_call(bwd))
    return out


def _stable(kind, one_round):
    p = PROTOCOL
    best = None
    for attempt in range(p.max_retries + 1):
        g = one_round()
        mean = statistics.mean(g)
        cv = statistics.pstdev(g) / mean if mean > 0 else float("inf")
        s = {"kind": kind, "geomeans_ms": g, "geomean_ms": _geomean(g), "cv": cv,
             "ok": cv <= p.cv_threshold, "attempts": attempt + 1}
        if best is None or cv < best["cv"]:
            best = s
        if s["ok"]:
            break
    return best


def _forward_stats(fn, inputs, params):
    p = PROTOCOL
    det = {k: v.detach() for k, v in inputs.items()}

    def call():
        with torch.no_grad():
            fn(det, params)

    return _stable("forward", lambda: [_geomean(_timings(call, p.warmup, p.iters))
                                       for _ in range(p.repeats)])


def _backward_stats(fn, inputs, params, grad_inputs, G):
    p = PROTOCOL

    def make_bwd():
        leaves = {}
        for k, v in inputs.items():
            t = v.detach().clone()
            if k in grad_inputs:
                t.requires_grad_(True)
            leaves[k] = t
        out = fn(leaves, params)
        return lambda: out.backward(G)

    return _stable("backward", lambda: [_geomean(_backward_timings(make_bwd, p.warmup, p.iters))
                                        for _ in range(p.repeats)])


def compare(case, candidate, device=None, seed=0, baseline=None):
    """Time ``candidate`` against ``torch.compile(case.reference_forward)`` (or ``baseline``)
    -> (report text, passed)."""
    p = PROTOCOL
    if device is None:
        device = "cuda" if torch.cuda.is_available() else "cpu"
    if device != "cuda":
        raise RuntimeError("timing needs a CUDA device")
    dtype = dtype_of(case.dtype)
    inputs = case.make_inputs(seed, dtype, device, requires_grad=False)
    with torch.no_grad():
        shape = case.reference_forward(inputs, case.params).shape
    G = torch.randn(shape, dtype=dtype, device=device,
                    generator=torch.Generator(device=device).manual_seed(777))
    base = baseline if baseline is not None else torch.compile(case.reference_forward)
    lines = [f"=== bench: case={case.name} (CUDA events, geometric means) ===",
             f"grad_inputs={case.grad_inputs} params={case.params} dtype={case.dtype}"]
    res = {}
    for name, fn in [("baseline(torch.compile)", base), ("candidate", candidate)]:
        f = _forward_stats(fn, inputs, case.params)
        b = _backward_stats(fn, inputs, case.params, case.grad_inputs, G)
        res[name] = (f, b)
        lines.append(f"\n[{name}]")
        for s in (f, b):
            lines.append(f"  {s['kind']:8s}: {s['geomean_ms']:.4f} ms  CV={s['cv'] * 100:.2f}%  "
                         f"x{s['attempts']}  {'ok' if s['ok'] else 'CV over threshold'}")
    (bf, bb), (cf, cb) = res["baseline(torch.compile)"], res["candidate"]
    fs, bs = bf["geomean_ms"] / cf["geomean_ms"], bb["geomean_ms"] / cb["geomean_ms"]
    lines.append("\n[speed-up candidate vs baseline]")
    lines.append(f"  forward : {fs:.4f}x (need >= {p.speedup_target}x) "
                 f"{'PASS' if fs >= p.speedup_target else 'FAIL'}")
    lines.append(f"  backward: {bs:.4f}x (need >= {p.speedup_target}x) "
                 f"{'PASS' if bs >= p.speedup_target else 'FAIL'}")
    cv_ok = all(s["ok"] for s in (bf, bb, cf, cb))
    passed = fs >= p.speedup_target and bs >= p.speedup_target and cv_ok
    if not cv_ok:
        lines.append("  CV over threshold: result void, re-measure")
    lines.append(f"\n=== gate: {'PASS' if passed else 'FAIL'} ===")
    return "\n".join(lines), passed
