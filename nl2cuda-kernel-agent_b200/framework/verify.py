"""Correctness gate (reference ``framework/verify.py:24-105``).

A candidate ``impl(inputs, params) -> output`` passes when, for every seed of the protocol,
its forward output and the gradient of every ``case.grad_inputs`` tensor match the case's
PyTorch reference within ``torch.allclose(atol, rtol)``.  The upstream gradient for seed ``s``
is drawn from ``torch.Generator(device).manual_seed(s + 10000)`` (reference verify.py:62) so
that reference and candidate see the same G.
"""
import torch

from framework.protocol import PROTOCOL, dtype_of


def _leaf_copies(inputs, grad_inputs):
    out = {}
    for name, t in inputs.items():
        c = t.detach().clone()
        if name in grad_inputs:
            c.requires_grad_(True)
        out[name] = c
    return out


def verify_forward(case, impl, device="cuda"):
    """Forward allclose over the protocol's seeds -> (ok, [(seed, ok, max_abs_err)])."""
    p = PROTOCOL
    dtype = dtype_of(case.dtype)
    rows = []
    for seed in p.seeds:
        inputs = case.make_inputs(seed, dtype, device, requires_grad=False)
        with torch.no_grad():
            want = case.reference_forward(inputs, case.params)
            got = impl(inputs, case.params)
        ok = bool(torch.allclose(got, want, atol=p.atol, rtol=p.rtol))
        rows.append((seed, ok, (got - want).abs().max().item() if want.numel() else 0.0))
    return all(r[1] for r in rows), rows


def verify_backward(case, impl, device="cuda"):
    """Per-input gradient allclose with a shared G -> (ok, [(seed, ok, {name: max_abs})])."""
    p = PROTOCOL
    dtype = dtype_of(case.dtype)
    rows = []
    for seed in p.seeds:
        base = case.make_inputs(seed, dtype, device, requires_grad=False)
        ref_in = _leaf_copies(base, case.grad_inputs)
        ref_out = case.reference_forward(ref_in, case.params)
        gen = torch.Generator(device=device).manual_seed(seed + 10_000)
        G = torch.randn(ref_out.shape, dtype=dtype, device=device, generator=gen)
        ref_out.backward(G)
        want = {k: ref_in[k].grad.detach().clone() for k in case.grad_inputs}

        imp_in = _leaf_copies(base, case.grad_inputs)
        impl(imp_in, case.params).backward(G.clone())

        oks, errs = {}, {}
        for k in case.grad_inputs:
            got = imp_in[k].grad
            oks[k] = bool(torch.allclose(got, want[k], atol=p.atol, rtol=p.rtol))
            errs[k] = (got - want[k]).abs().max().item() if got.numel() else 0.0
        rows.append((seed, all(oks.values()), errs))
    return all(r[1] for r in rows), rows


def verify_all(case, impl, device=None):
    """Forward + backward gate -> (ok, report text)."""
    if device is None:
        device = "cuda" if torch.cuda.is_available() else "cpu"
    lines = [f"=== verify: case={case.name} (device={device}) ===",
             f"grad_inputs={case.grad_inputs} params={case.params} dtype={case.dtype}"]
    fwd_ok, fwd = verify_forward(case, impl, device)
    lines.append(f"\n[forward] {'PASS' if fwd_ok else 'FAIL'}")
    for seed, ok, err in fwd:
        lines.append(f"  seed={seed}: {'ok' if ok else 'X'}  max_abs_err={err:.3e}")
    bwd_ok, bwd = verify_backward(case, impl, device)
    lines.append(f"\n[backward] {'PASS' if bwd_ok else 'FAIL'}")
    for seed, ok, errs in bwd:
        e = " ".join(f"d{k}_err={v:.3e}" for k, v in errs.items())
        lines.append(f"  seed={seed}: {'ok' if ok else 'X'}  {e}")
    ok = fwd_ok and bwd_ok
    lines.append(f"\n=== overall: {'PASS' if ok else 'FAIL'} ===")
    return ok, "\n".join(lines)
