"""Profile a case candidate: where the CUDA time goes, and what ncu's counters say.

The reference's ``skill/scripts/profile_case.py`` prints torch.profiler's kernel table for a
case candidate (forward, backward or both).  This tool keeps that use, and adds a summariser for
Nsight Compute output, so that a run on the GPU box turns into the figures a roofline needs:

    python -m framework.profile --case rbf [--impl cases.rbf.op:candidate] [--mode both]
        torch.profiler table of the candidate's kernels, and CUDA time vs wall time

    python -m framework.profile --ncu-commands --case rbf
        the two ncu command lines to run on one GPU (launch list; sections of the top kernels),
        both with --clock-control none

    python -m framework.profile --launches launches.csv
        per-kernel launches, total and mean time and share, from a
        ``--metrics gpu__time_duration.sum --csv`` launch list

    python -m framework.profile --raw raw.csv
        per-kernel DRAM bytes, DRAM and tensor-pipe utilisation, issue rate and top stall
        reasons, from ``ncu -i report.ncu-rep --page raw --csv``

Run it from the package directory (``nl2cuda-kernel-agent_b200``) or with it on ``sys.path``.
"""
import argparse
import collections
import csv
import importlib
import io
import os
import sys
import time

_HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if _HERE not in sys.path:
    sys.path.insert(0, _HERE)


# ----------------------------------------------------------------------------- ncu CSV parsing

def _csv_rows(text):
    """Rows of an ncu CSV log, skipping the ==PROF== / ==WARNING== lines ncu interleaves."""
    lines = [ln for ln in text.splitlines() if ln.startswith('"')]
    return list(csv.reader(io.StringIO("\n".join(lines))))


def _to_us(value, unit):
    v = float(str(value).replace(",", ""))
    unit = (unit or "").strip()
    scale = {"ns": 1e-3, "nsecond": 1e-3, "us": 1.0, "usecond": 1.0, "ms": 1e3, "msecond": 1e3,
             "s": 1e6, "second": 1e6}
    if unit not in scale:
        raise ValueError(f"unknown time unit {unit!r}")
    return v * scale[unit]


def summarize_launches(text, name_width=60):
    """[(kernel, launches, total_us, mean_us, share)] from a launch-list CSV, largest first."""
    rows = _csv_rows(text)
    if not rows:
        return []
    hdr = rows[0]
    ki, vi, ui = hdr.index("Kernel Name"), hdr.index("Metric Value"), hdr.index("Metric Unit")
    mi = hdr.index("Metric Name")
    agg = collections.OrderedDict()
    for r in rows[1:]:
        if len(r) <= max(ki, vi, ui, mi) or r[mi] != "gpu__time_duration.sum":
            continue
        k = r[ki][:name_width]
        a = agg.setdefault(k, [0, 0.0])
        a[0] += 1
        a[1] += _to_us(r[vi], r[ui])
    total = sum(t for _, t in agg.values()) or 1.0
    out = [(k, n, t, t / n, t / total) for k, (n, t) in agg.items()]
    return sorted(out, key=lambda x: -x[2])


_RAW_KEYS = {
    "duration_us": "gpu__time_duration.sum",
    "dram_read": "dram__bytes_read.sum",
    "dram_write": "dram__bytes_write.sum",
    "dram_pct": "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed",
    "tensor_pct": "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed",
    "issue": "smsp__issue_active.avg.per_cycle_active",
    "registers": "launch__registers_per_thread",
}
_BYTES = {"byte": 1.0, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9}


def summarize_raw(text, name_width=60):
    """Per captured launch: the roofline counters and the top stall reasons, from
    ``ncu -i ... --page raw --csv`` (first row: names, second row: units)."""
    rows = _csv_rows(text)
    if len(rows) < 3:
        return []
    hdr, units = rows[0], rows[1]
    out = []
    for r in rows[2:]:
        rec = {"kernel": r[hdr.index("Kernel Name")][:name_width]}
        for key, metric in _RAW_KEYS.items():
            if metric not in hdr:
                continue
            i = hdr.index(metric)
            if i >= len(r) or r[i] in ("", "n/a"):
                continue
            v = float(r[i].replace(",", ""))
            u = units[i]
            if u in _BYTES:
                v *= _BYTES[u]
            elif key == "duration_us":
                v = _to_us(v, u)
            rec[key] = v
        stalls = []
        for i, m in enumerate(hdr):
            if (m.startswith("smsp__average_warps_issue_stalled_")
                    and m.endswith("_per_issue_active.ratio") and i < len(r)
                    and r[i] not in ("", "n/a")):
                name = m[len("smsp__average_warps_issue_stalled_"):-len("_per_issue_active.ratio")]
                stalls.append((float(r[i].replace(",", "")), name))
        rec["stalls"] = [(n, v) for v, n in sorted(stalls, reverse=True)[:5]]
        out.append(rec)
    return out


def format_launches(summary):
    lines = [f"{'launches':>8} {'total us':>10} {'mean us':>9} {'share':>6}  kernel"]
    for k, n, t, m, sh in summary:
        lines.append(f"{n:8d} {t:10.1f} {m:9.2f} {100 * sh:5.1f}%  {k}")
    return "\n".join(lines)


def format_raw(recs):
    lines = []
    for r in recs:
        lines.append(r["kernel"])
        if "duration_us" in r:
            lines.append(f"  duration {r['duration_us']:.2f} us")
        if "dram_read" in r or "dram_write" in r:
            rd, wr = r.get("dram_read", 0.0), r.get("dram_write", 0.0)
            lines.append(f"  dram read {rd / 1e6:.2f} MB, write {wr / 1e6:.2f} MB, "
                         f"traffic {(rd + wr) / 1e6:.2f} MB")
        for key, label in (("dram_pct", "dram throughput %"), ("tensor_pct", "tensor pipe %"),
                           ("issue", "issue active / cycle"), ("registers", "registers")):
            if key in r:
                lines.append(f"  {label} {r[key]:.2f}")
        if r["stalls"]:
            lines.append("  stalls / issue: " + ", ".join(f"{n} {v:.2f}" for n, v in r["stalls"]))
    return "\n".join(lines)


# The kernels worth a full capture, per case: one `ncu` command each, filtered to that kernel.
CAPTURE_KERNELS = {
    "rbf": ("rbf_fwd_tc_kernel", "rbf_bwd_tc_kernel"),
    "cosine_sim": ("rbf_fwd_tc_kernel", "rbf_bwd_tc_kernel"),
}


def ncu_commands(case, impl, py="python", kernels=None):
    """The capture commands for one GPU: the plain run (which must exit 0 first), the launch
    list, and one section capture per kernel (`-k regex:<kernel>`, three launches at most) on the
    case's own small size (a few GB on the device at most)."""
    run = f"{py} -m framework.profile --case {case}" + (f" --impl {impl}" if impl else "")
    cmds = [
        f"{run} && ncu --metrics gpu__time_duration.sum --clock-control none --csv "
        f"--log-file launches.csv {run}",
    ]
    for k in (kernels or CAPTURE_KERNELS.get(case, ("rbf_bwd_tc_kernel",))):
        cmds.append(
            f"{run} && ncu -k regex:{k} -c 3 --section SpeedOfLight "
            f"--section MemoryWorkloadAnalysis --section WarpStateStats "
            f"--metrics dram__bytes_read.sum,dram__bytes_write.sum,"
            f"sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed "
            f"--clock-control none -o prof_{k} {run}")
        cmds.append(f"ncu -i prof_{k}.ncu-rep --page raw --csv > raw_{k}.csv")
    return cmds


# ----------------------------------------------------------------------------- torch.profiler

def _load_case(name):
    return importlib.import_module(f"cases.{name}").CASE


def _load_impl(spec):
    mod, fn = spec.split(":")
    return getattr(importlib.import_module(mod), fn)


def profile_candidate(case_name, impl=None, mode="both", iters=20, seed=0):
    """torch.profiler table of the candidate's CUDA kernels, plus CUDA time vs wall time."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    from framework.protocol import dtype_of
    case = _load_case(case_name)
    fn = _load_impl(impl) if impl else _load_impl(f"cases.{case_name}.op:candidate")
    dev = torch.device("cuda")
    inputs = case.make_inputs(seed, dtype_of(case.dtype), dev, requires_grad=mode != "forward")
    params = dict(case.params)

    def once():
        out = fn(inputs, params)
        if mode != "forward":
            out.backward(torch.ones_like(out) if mode == "backward" else torch.randn_like(out))
            for v in inputs.values():
                v.grad = None
        return out

    for _ in range(3):
        once()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA], acc_events=True) as prof:
        t0 = time.perf_counter()
        for _ in range(iters):
            once()
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
    table = prof.key_averages().table(sort_by="cuda_time_total", row_limit=15)
    cuda_us = sum(e.self_device_time_total for e in prof.key_averages()) / iters
    return table, cuda_us, wall / iters * 1e6


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--case")
    ap.add_argument("--impl", default=None)
    ap.add_argument("--mode", choices=["forward", "backward", "both"], default="both")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--launches", help="summarise an ncu launch-list CSV")
    ap.add_argument("--raw", help="summarise an ncu --page raw --csv export")
    ap.add_argument("--ncu-commands", action="store_true", help="print the capture commands")
    args = ap.parse_args(argv)
    if args.launches:
        with open(args.launches) as f:
            print(format_launches(summarize_launches(f.read())))
        return 0
    if args.raw:
        with open(args.raw) as f:
            print(format_raw(summarize_raw(f.read())))
        return 0
    if not args.case:
        ap.error("--case is required (or --launches / --raw)")
    if args.ncu_commands:
        print("\n".join(ncu_commands(args.case, args.impl)))
        return 0
    table, cuda_us, wall_us = profile_candidate(args.case, args.impl, args.mode, args.iters)
    print(table)
    print(f"per iteration: CUDA kernel time {cuda_us:.1f} us, wall time {wall_us:.1f} us "
          f"({100 * cuda_us / max(wall_us, 1e-9):.0f}% of wall on the device)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
