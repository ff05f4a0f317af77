#!/usr/bin/env python
"""RBF kernel matrix forward + backward on B200: the headline benchmark.

Metric: RBF fwd+bwd ms, GFLOP/s and % roofline at N=M=4096, D=64, with
1/2/4/8-GPU scaling.  One "step" = forward K = rbf(X, Y) + backward (dX, dY) from an upstream
gradient G, fp32 in and out.  FLOP per step = 6*N*M*D; algorithmic HBM bytes per step =
12*N*M + 12*(N+M)*D.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c1]
                  [--scaling weak|strong]

N = 1 runs config c1 (N=M=4096, D=64); --config c0..c4 picks another BASELINE configuration.
Under torchrun (WORLD_SIZE = N > 1) the work is sharded by rows of X (and of G, K) with Y
replicated.  --scaling weak (the default): every rank owns the config's N rows ("scaling":
"weak").  --scaling strong: the config's N rows are split across the ranks, so the same problem
is solved at every N (the c4 1->8 GPU target: --config c4 --scaling strong).  The partial dY is
reduced over NVLink peer memory by this library (the dY partials go into the rank's slot of a
symmetric buffer, then one bounded cross-GPU barrier and a gather) up to 4 ranks while dY is
small, and with one NCCL all-reduce otherwise, where that measured faster (RBF_DY_REDUCE=peer or
nccl forces either).  After timing, every rank checks sampled rows of K and dX and columns of dY
of one more step against the CPU oracle ("parity" in the JSON line).
``value`` = whole-job GFLOP/s = (6 * N_global * M * D) / (max over ranks of the device time of
one step).  The step is ``shard.forward_backward_shard``: the library's one-call forward +
backward (rbf_sm100_forward_backward) plus the dY reduction when N > 1.  Inputs are resident in
HBM when timing starts; L2 is flushed before every timed step, outside the events: a 256 MiB
write, then a 256 MiB read of a second buffer, so that the flush's own dirty lines are written
back before the step rather than during it.  With N > 1 a 4-byte all-reduce after the flush
lines the ranks up again before the start event.  Besides the step, the line carries the
forward (``ms_fwd``), the backward (``ms_bwd``) and the one-call forward + backward
(``ms_fused``), each replayed alone from its own CUDA graph.

``--impl reference`` times the reference's own CPU implementation of the path (its broadcast
``reference.py`` forward + torch autograd, restated in oracle/reference_port.py) on the host
cores, on a bounded sample of rows per step, and prints the same JSON line with
"impl": "reference".  Under torchrun only rank 0 runs it.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "nl2cuda-kernel-agent_b200")
for _p in (PKG, ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "RBF fwd+bwd ms, GFLOP/s and % roofline at N=M=4096 D=64; 1/2/4/8 GPU scaling"
UNIT = "GFLOP/s"
L2_FLUSH_BYTES = 256 << 20


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--config", default="c1", help="c0..c4 (cases/rbf/config.py CONFIGS)")
    ap.add_argument("--scaling", choices=("weak", "strong"), default="weak",
                    help="weak: every rank owns the config's N rows (N_global = N * world); "
                         "strong: the config's N rows are split across the ranks")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the post-timing oracle spot check of sampled rows / columns")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0,
                    help="target CPU seconds of the cpu_baseline sample")
    ap.add_argument("--case", choices=("rbf", "cosine_sim"), default="rbf",
                    help="rbf (the headline) or the cosine-similarity case (one GPU)")
    ap.add_argument("--cos-size", type=int, default=4096,
                    help="N = M of the cosine-similarity workload (D = 64)")
    return ap.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])),
                "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
                "source": "fallback"}


def traffic_table():
    """dram__bytes_read.sum + dram__bytes_write.sum per launch, from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


class ClockSampler:
    """SM clock and throttle reasons sampled while the timed region runs: through NVML every
    ~0.5 ms (the timed region lasts milliseconds), else nvidia-smi every 200 ms.  Read-only."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    # NVML clocks-event (throttle) reason bits
    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
                   "hw_thermal_slowdown": 0x40}

    def __init__(self, gpu_id, period_s=0.0005):
        self.gpu_id = gpu_id
        self.period_s = period_s
        self.proc = None
        self.lines = []
        self.thread = None
        self.nvml = None
        self.samples = []  # (sm_mhz, reason bits) from NVML
        self.max_mhz = None
        self.running = False

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            gid = str(self.gpu_id)
            h = (pynvml.nvmlDeviceGetHandleByUUID(gid) if gid.startswith("GPU-")
                 else pynvml.nvmlDeviceGetHandleByIndex(int(gid)))
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                getattr(pynvml, "nvmlDeviceGetCurrentClocksThrottleReasons")
            self.nvml = (pynvml, h, reasons)
        except Exception:
            self.nvml = None
        if self.nvml is not None:
            self.running = True
            # The timed region lasts milliseconds: let the polling thread take the interpreter
            # often enough (the default switch interval is 5 ms).
            self.switch = sys.getswitchinterval()
            sys.setswitchinterval(1e-4)
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            return
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu_id), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _poll(self):
        pynvml, h, reasons = self.nvml
        while self.running:
            try:
                self.samples.append((float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)),
                                     int(reasons(h))))
            except Exception:
                return
            time.sleep(self.period_s)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.nvml is not None:
            self.running = False
            if self.thread:
                self.thread.join(timeout=2)
            sys.setswitchinterval(self.switch)
            if not self.samples:
                return None
            names = sorted(n for n, bit in self.REASON_BITS.items()
                           if any(r & bit for _, r in self.samples))
            return {"sm_mhz": statistics.median(s for s, _ in self.samples),
                    "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples),
                    "source": "nvml"}
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for n, v in zip(names, parts[3:7]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvidia-smi"}


class L2Flush:
    """Evicts L2 between timed steps.  A write larger than L2 evicts the inputs but leaves
    ~L2-size of dirty lines whose write-back would land inside the next timed region (measured:
    plain TMA reads of G and K at c1 ran at 4.1 TB/s after a write flush, 4.7 TB/s after write +
    read); reading a second buffer larger than L2 evicts those too."""

    def __init__(self, dev):
        import torch
        self.torch = torch
        self.w = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
        self.r = torch.zeros(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
        self.sink = torch.zeros((), dtype=torch.float32, device=dev)

    def __call__(self):
        self.w.zero_()
        self.torch.sum(self.r, dim=0, out=self.sink)


def nvsmi_id(device):
    import torch
    try:
        return "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
    except Exception:
        return device.index if device.index is not None else 0


def workload(cfg_name, world, rank=0, scaling="weak"):
    """The config's shapes and this rank's rows.  weak: every rank owns N rows (N_global =
    N * world); strong: the config's N rows are split by shard.row_range."""
    from cases.rbf import config
    c = dict(config.CONFIGS[cfg_name])
    if scaling == "strong":
        from cases.rbf import shard
        c["N_global"] = c["N"]
        c["row0"], row1 = shard.row_range(c["N"], world, rank)
        c["rows_per_rank"] = row1 - c["row0"]
    else:
        c["N_global"] = c["N"] * world
        c["row0"] = rank * c["N"]
        c["rows_per_rank"] = c["N"]
    return c


def run_reference(args, world, rank):
    """The reference's CPU implementation (oracle/reference_port.py) on this host's cores.

    Where the whole workload fits (the [N, M, D] broadcast intermediate of reference.py and its
    autograd buffers within a third of the available host memory, and one step within ~20 s of
    CPU time, e.g. c0 and c1 on a many-core host) every step is the reference's forward +
    backward over ALL rows, as written.  Otherwise a step is a bounded sample of rows of X
    against all of Y, and ms_per_step scales it linearly to all N rows."""
    if rank != 0:
        return
    import torch
    from oracle import reference_port
    c = workload(args.config, world, 0, args.scaling)
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    N, M, D, g = c["N_global"], c["M"], c["D"], c["gamma"]
    probe_s, probe_rows = reference_port.time_sample(N, M, D, g, 32, threads)
    per_row_s = probe_s / max(probe_rows, 1)
    try:
        import psutil
        avail = psutil.virtual_memory().available
    except Exception:  # pragma: no cover
        avail = 0
    full_bytes = 4 * 4 * N * M * D  # diff, diff**2 and their autograd grads, fp32
    verbatim = full_bytes < avail / 3 and per_row_s * N < 20.0
    if verbatim:
        rows = N
    else:
        # One step = a bounded sample of rows of X against all of Y, ~1 s of CPU work.
        rows = int(max(8, min(N, 32 * max(1.0, 1.0 / max(probe_s, 1e-3)))))
    gen = torch.Generator().manual_seed(0)
    X = torch.randn(rows, D, generator=gen)
    Y = torch.randn(M, D, generator=gen)
    G = torch.randn(rows, M, generator=gen)
    block = rows if verbatim else 256
    for _ in range(args.warmup):
        reference_port.forward_backward(X, Y, G, g, block_rows=block)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        reference_port.forward_backward(X, Y, G, g, block_rows=block)
        times.append(time.perf_counter() - t0)
    per_row = statistics.mean(times) / rows
    ms_step = per_row * N * 1e3
    gflops = 6.0 * rows * M * D / statistics.mean(times) / 1e9
    if verbatim:
        sample = f"all {N} rows of X x all {M} rows of Y, fwd+bwd, per step (reference.py as written)"
        extrap = "none: every step runs the whole workload"
    else:
        sample = f"{rows} rows of X x all {M} rows of Y, fwd+bwd, per step"
        extrap = "ms_per_step scales the sample linearly to all N rows"
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gflops, 3), "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_step, 3), "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{args.config}: RBF fwd+bwd N={N} M={M} D={D} gamma={g:.6g}",
                   "N": N, "M": M, "D": D, "sample_rows_per_step": rows,
                   "extrapolation": extrap},
        "cpu_baseline": {"value": round(gflops, 3), "unit": UNIT, "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(gflops, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline(c, seconds):
    import torch
    from oracle import reference_port
    threads = os.cpu_count() or 1
    N, M, D, g = c["N_global"], c["M"], c["D"], c["gamma"]
    probe_s, _ = reference_port.time_sample(N, M, D, g, 16, threads)
    rows = int(max(16, min(N, 16 * seconds / max(probe_s, 1e-3) / 2)))
    # Repeat the sample (at most all N rows per pass) until about `seconds` of CPU work.
    sec, done = reference_port.time_sample(N, M, D, g, rows, threads, min_seconds=0.75 * seconds)
    torch.set_num_threads(threads)
    return {"value": round(6.0 * done * M * D / sec / 1e9, 3), "unit": UNIT, "cores": threads,
            "kind": "port",
            "sample": f"{done} rows of X ({rows} per pass, of {N}) x all {M} rows of Y, "
                      f"fwd+bwd ({sec:.1f} s on {threads} threads)"}


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.case == "cosine_sim":
        if world > 1:
            raise SystemExit("--case cosine_sim runs on one GPU")
        run_cosine(args)
        return
    if args.impl == "reference":
        run_reference(args, world, rank)
        return

    import torch
    import torch.distributed as dist
    from cases.rbf import native, op, shard
    from cases.rbf.reference import draw

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    c = workload(args.config, world, rank, args.scaling)
    n, M, D, g = c["rows_per_rank"], c["M"], c["D"], c["gamma"]
    Ng, row0 = c["N_global"], c["row0"]

    # Inputs: this rank's rows of X (and of G), Y replicated; resident in HBM.  X is drawn for
    # all N_global rows from one seed, so a strong-scaling run at any world size solves the
    # same X, Y.
    X_all, Y = draw(1234, torch.float32, dev, Ng, M, D, c["ydist"], c["xscale"])
    X = X_all[row0:row0 + n].contiguous()
    del X_all
    G = torch.randn(n, M, dtype=torch.float32, device=dev,
                    generator=torch.Generator(device=dev).manual_seed(777 + rank))
    flush_l2 = L2Flush(dev)
    compute = shard.NativeShardCompute()
    route = None
    dy_reduce = "none"
    if world > 1:
        # auto: the library's NVLink peer exchange up to 4 ranks, where it measured faster than
        # NCCL (109.5 vs 115.5 us per step at 2 GPUs, 115.7 vs 119.2 at 4); NCCL at 8 (129.5 vs
        # 133.5 us: every rank then reads 7 MB of partials).
        # A large dY (c4: 64 MB) goes to NCCL at every N: the one-phase peer sum reads every
        # rank's whole partial.
        dy_reduce = os.environ.get("RBF_DY_REDUCE", "auto")
        if dy_reduce == "auto":
            dy_reduce = "peer" if world <= 4 and M * D * 4 <= (8 << 20) else "nccl"
        if dy_reduce == "peer":
            route = shard.RoutedDy(M, D, dev)

    def step():
        return shard.forward_backward_shard(X, Y, G, g, compute=compute, route=route)

    for _ in range(max(args.warmup, 0)):
        step()
    torch.cuda.synchronize()

    # The timed step is replayed from a CUDA graph: the host work of the Python binding (tens of
    # microseconds per call) stays out of the device timeline.  The graph holds every kernel and
    # memset of one forward + backward (+ the NCCL all-reduce when N > 1).
    def capture(fn):
        gr = torch.cuda.CUDAGraph()
        before = native.launch_count()
        with torch.cuda.graph(gr):
            fn()
        return gr, native.launch_count() - before

    step_graph, launches_per_step = capture(step)
    for _ in range(max(args.warmup, 0)):
        step_graph.replay()
    torch.cuda.synchronize()

    sampler = ClockSampler(nvsmi_id(dev))
    sampler.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    # N > 1: after each rank's L2 flush, a 4-byte all-reduce lines the ranks up again before the
    # start event.  The flush's read pass takes a different time on each GPU; without this, a
    # rank that finished its flush early would count its wait for the others inside the step's
    # dY reduction (measured at 2 GPUs: 124-183 us per step instead of 106-112 us).
    align = torch.zeros(1, dtype=torch.float32, device=dev) if world > 1 else None
    evs = []
    for _ in range(args.steps):
        flush_l2()
        if align is not None:
            dist.all_reduce(align)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        step_graph.replay()
        b.record(stream)
        evs.append((a, b))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    launches = launches_per_step * args.steps
    clocks = sampler.stop()
    step_ms = [a.elapsed_time(b) for a, b in evs]
    ms_local = statistics.mean(step_ms)
    ms = shard.max_over_ranks(ms_local, device=dev)

    # Dominant-kernel roofline: the forward (split pass + kernel) and the backward kernel, each
    # replayed alone from its own graph, timed with events on the launching stream.
    def time_alone(gr, reps):
        out = []
        for _ in range(reps):
            flush_l2()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            gr.replay()
            b.record(stream)
            out.append((a, b))
        torch.cuda.synchronize()
        return statistics.mean(a.elapsed_time(b) for a, b in out)

    K, ws = native.forward_with_workspace(X, Y, g)
    torch.cuda.synchronize()
    fwd_graph, _ = capture(lambda: native.forward_with_workspace(X, Y, g))
    bwd_graph, _ = capture(lambda: native.rbf_backward(X, Y, G, K, g, workspace=ws))
    reps = max(args.steps, 5)
    ms_fwd = time_alone(fwd_graph, reps)
    ms_bwd = time_alone(bwd_graph, reps)
    # The one-call forward + backward (rbf_sm100_forward_backward): this rank's step without
    # the dY reduction.
    fused_graph, _ = capture(lambda: native.rbf_forward_backward(X, Y, G, g))
    ms_fused = time_alone(fused_graph, reps)
    pk = peaks()
    fwd_bytes = 4 * n * M + 4 * (n + M) * D
    bwd_bytes = 8 * n * M + 8 * (n + M) * D
    bwd_flop = 4 * n * M * D
    if ms_bwd >= ms_fwd:
        kname, kms, kbytes = "rbf backward (prepared)", ms_bwd, bwd_bytes
    else:
        kname, kms, kbytes = "rbf forward (split + kernel)", ms_fwd, fwd_bytes
    achieved = kbytes / (kms * 1e-3) / 1e9
    tr = traffic_table().get(f"{kname}|{args.config}")
    roofline = {"kernel": kname, "bound": "hbm", "achieved": round(achieved, 1),
                "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4),
                "traffic": tr, "peak_source": pk["source"],
                "algorithmic_bytes_per_launch": kbytes, "ms_per_launch": round(kms, 5)}

    # Whole-step roofline (BASELINE's % roofline): max(FLOP / P_tf32, bytes / HBM).
    flop = 6.0 * Ng * M * D
    p_tf32 = pk["bf16_tflops"] / 2.0 * 1e12
    t_tc = 6.0 * n * M * D / p_tf32
    t_hbm = (12.0 * n * M + 12.0 * (n + M) * D) / (pk["hbm_gbs"] * 1e9)
    t_roof = max(t_tc, t_hbm)
    gflops = flop / (ms * 1e-3) / 1e9

    # End to end through the public API with host buffers (skipped where one step would copy
    # more than 4 GiB over PCIe: c2-c4 move 2-32 GiB of K and G per step, which the host link,
    # not the kernels, would time).
    e2e, e2e_skipped = None, None
    if args.no_e2e:
        e2e_skipped = "--no-e2e"
    elif 8 * n * M > (4 << 30):
        e2e_skipped = f"host copies of {8 * n * M / 2**30:.1f} GiB per step (K out, G in)"
    else:
        e2e = run_e2e(X, Y, G, g, world, dev, args, shard, op, route)

    # Parity of this very run, after timing: sampled K and dX rows of every rank, and dY
    # columns (each rank's fp64 oracle partial over its rows, summed across ranks) against the
    # CPU oracle under the 1e-3 gate.  The oracle is imported only here.
    parity = None
    if not args.no_parity:
        parity = spot_check(X, Y, G, g, step, world, dev, shard)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(c, args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(gflops, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
            "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic (seeded X, Y, G with the config's distributions)",
            "config": {"workload": f"{args.config}: RBF fwd+bwd fp32, {n} rows of X per rank "
                                   f"(N={Ng} total, {args.scaling} scaling), M={M}, D={D}, "
                                   f"gamma={g:.6g}",
                       "N": Ng, "M": M, "D": D, "rows_per_rank": n,
                       "l2": "flushed before every timed step (256 MiB write + 256 MiB read, outside events)",
                       "parallelism": f"row-shard x{world}" + (
                           ", dY reduced in the backward over NVLink peer memory"
                           if dy_reduce == "peer" else ", dY all-reduce (NCCL)"
                           if world > 1 else "")},
            "ms_fwd": round(ms_fwd, 5), "ms_bwd": round(ms_bwd, 5),
            "ms_fused": round(ms_fused, 5),
            "pct_roofline_step": round(100.0 * t_roof / (ms * 1e-3), 2),
            "roofline_step_us": round(t_roof * 1e6, 2),
            "roofline": roofline,
            "gpu_launches": int(launches),
            "clocks": clocks,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "parity": parity,
        }
        if e2e_skipped:
            line["e2e_skipped"] = e2e_skipped
        print(json.dumps(line), flush=True)
    # Graphs that captured NCCL work must be gone before the communicator is; the process then
    # exits without tearing the process group down (destroying it while captured collectives
    # existed hung on this pool).
    del step_graph, fwd_graph, bwd_graph
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        sys.stdout.flush()
        sys.stderr.flush()
        os._exit(0)


def spot_check(X, Y, G, gamma, step, world, dev, shard, n_rows=8, n_cols=8, seed=5):
    """Max errors of one untimed step against the CPU oracle on sampled rows / columns."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from oracle import oracle
    K, dX, dY = step()
    torch.cuda.synchronize()
    n, M = G.shape
    rng = np.random.default_rng(seed)
    rows = np.unique(np.concatenate([[0, n - 1], rng.integers(0, n, n_rows)])) if n else \
        np.zeros(0, np.int64)
    cols = np.unique(np.concatenate([[0, M - 1], rng.integers(0, M, n_cols)]))
    ri = torch.from_numpy(rows).to(dev)
    ci = torch.from_numpy(cols).to(dev)
    Xh, Yh = X.cpu().numpy(), Y.cpu().numpy()
    k_ref = oracle.forward_rows(Xh, Yh, gamma, rows)
    dx_ref = oracle.dx_rows(Xh[rows], Yh, G.index_select(0, ri).cpu().numpy(), gamma,
                            np.arange(len(rows)))
    dy_part = oracle.dy_cols(Xh, Yh[cols], G.index_select(1, ci).cpu().numpy(), gamma,
                             np.arange(len(cols)))
    dy_ref = torch.from_numpy(dy_part).to(dev)
    if world > 1:
        dist.all_reduce(dy_ref)  # fp64 sum of every rank's oracle partial
    dy_ref = dy_ref.cpu().numpy()
    out = {}
    ok = True
    for name, got, ref in (("K", K.index_select(0, ri).cpu().numpy(), k_ref),
                           ("dX", dX.index_select(0, ri).cpu().numpy(), dx_ref),
                           ("dY", dY.index_select(0, ci).cpu().numpy(), dy_ref)):
        err = np.abs(got.astype(np.float64) - ref)
        mabs = float(err.max()) if err.size else 0.0
        mrel = float((err / np.maximum(np.abs(ref), 1e-6)).max()) if err.size else 0.0
        ok = ok and bool(np.all(err <= 1e-3 + 1e-3 * np.abs(ref)))
        out[name] = [shard.max_over_ranks(mabs, device=dev), shard.max_over_ranks(mrel, device=dev)]
    ok = shard.max_over_ranks(0.0 if ok else 1.0, device=dev) == 0.0
    return {"max_abs": max(v[0] for v in out.values()),
            "per_output_max_abs_rel": out, "gate_1e-3": ok,
            "sample": f"{len(rows)} rows of K and dX per rank, {len(cols)} columns of dY, "
                      "vs the fp64 CPU oracle, after timing"}


COS_METRIC = "cosine_sim fwd+bwd GFLOP/s at N=M={n} D=64 (one GPU)"


def run_cosine(args):
    """The cosine-similarity case on one GPU: one step = forward S = cos(A, B) + backward
    (dA, dB) from an upstream dS, fp32.  FLOP per step = 6*N*M*D; algorithmic HBM bytes per step
    = 8*N*M + 16*(N+M)*D (S written, dS read, rows and gradients).  Same timing rules as the RBF
    bench (CUDA graph, L2 flushed outside the events, NVML clocks)."""
    import torch
    from cases.cosine_sim import config as cos_config
    from cases.cosine_sim import native as cnative
    from cases.cosine_sim import op as cop
    from cases.rbf import native

    n = M = args.cos_size
    D, eps = 64, cos_config.EPS
    metric = COS_METRIC.format(n=n)
    workload_name = f"cosine_sim fwd+bwd fp32, N=M={n}, D={D}, eps={eps:g}"
    if args.impl == "reference":
        from oracle import reference_port
        threads = os.cpu_count() or 1
        sec, done = reference_port.cos_time_sample(n, M, D, eps, 256, threads,
                                                   min_seconds=max(1.0, args.cpu_seconds / 4))
        gf = 6.0 * done * M * D / sec / 1e9
        print(json.dumps({
            "impl": "reference", "metric": metric, "value": round(gf, 3), "unit": UNIT,
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(sec / done * n * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": workload_name, "N": n, "M": M, "D": D},
            "cpu_baseline": {"value": round(gf, 3), "unit": UNIT, "cores": threads,
                             "kind": "port", "sample": f"{done} rows of A x all {M} rows of B"},
            "e2e": {"value": round(gf, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}), flush=True)
        return

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev).manual_seed(4321)
    A = torch.randn(n, D, device=dev, generator=gen)
    B = torch.randn(M, D, device=dev, generator=gen)
    dS = torch.randn(n, M, device=dev, generator=gen)
    flush_l2 = L2Flush(dev)

    def fwd():
        return cnative.forward_with_workspace(A, B, eps)

    _, ws = fwd()  # the workspace the backward graph reads

    def bwd():
        return cnative.cos_backward(dS, n, M, D, eps, workspace=ws)

    def step_fb():
        _, ws_step = cnative.forward_with_workspace(A, B, eps)
        cnative.cos_backward(dS, n, M, D, eps, workspace=ws_step)

    for _ in range(max(args.warmup, 0)):
        step_fb()
    torch.cuda.synchronize()

    def capture(fn):
        gr = torch.cuda.CUDAGraph()
        before = native.launch_count()
        with torch.cuda.graph(gr):
            fn()
        return gr, native.launch_count() - before

    step_graph, launches_per_step = capture(step_fb)
    fwd_graph, _ = capture(fwd)
    bwd_graph, _ = capture(bwd)
    for _ in range(max(args.warmup, 0)):
        step_graph.replay()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)

    def time_graph(gr, reps):
        evs = []
        for _ in range(reps):
            flush_l2()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            gr.replay()
            b.record(stream)
            evs.append((a, b))
        torch.cuda.synchronize()
        return statistics.mean(a.elapsed_time(b) for a, b in evs)

    sampler = ClockSampler(nvsmi_id(dev))
    sampler.start()
    ms = time_graph(step_graph, args.steps)
    clocks = sampler.stop()
    reps = max(args.steps, 5)
    ms_fwd = time_graph(fwd_graph, reps)
    ms_bwd = time_graph(bwd_graph, reps)

    pk = peaks()
    fwd_bytes = 4 * n * M + 4 * (n + M) * D
    bwd_bytes = 4 * n * M + 12 * (n + M) * D
    if ms_bwd >= ms_fwd:
        kname, kms, kbytes = "cosine backward (prepared)", ms_bwd, bwd_bytes
    else:
        kname, kms, kbytes = "cosine forward (normalise + kernel)", ms_fwd, fwd_bytes
    achieved = kbytes / (kms * 1e-3) / 1e9
    roofline = {"kernel": kname, "bound": "hbm", "achieved": round(achieved, 1),
                "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4),
                "traffic": traffic_table().get(f"{kname}|cos{n}"), "peak_source": pk["source"],
                "algorithmic_bytes_per_launch": kbytes, "ms_per_launch": round(kms, 5)}
    t_roof = max(6.0 * n * M * D / (pk["bf16_tflops"] / 2.0 * 1e12),
                 cos_config.hbm_bytes(n, M, D) / (pk["hbm_gbs"] * 1e9))
    gflops = 6.0 * n * M * D / (ms * 1e-3) / 1e9

    # End to end through the autograd op with pinned host buffers (dS copied in on a side stream
    # during the forward, S copied out on another during the backward).
    Ah, Bh, dSh = A.cpu().pin_memory(), B.cpu().pin_memory(), dS.cpu().pin_memory()
    Sh = torch.empty(n, M).pin_memory()
    dAh, dBh = torch.empty(n, D).pin_memory(), torch.empty(M, D).pin_memory()
    h2d, d2h = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)

    def e2e_once():
        Ad = Ah.to(dev, non_blocking=True).requires_grad_(True)
        Bd = Bh.to(dev, non_blocking=True).requires_grad_(True)
        h2d.wait_stream(stream)
        with torch.cuda.stream(h2d):
            dSd = dSh.to(dev, non_blocking=True)
        dSd.record_stream(stream)
        Sd = cop.candidate({"A": Ad, "B": Bd}, {"eps": eps})
        d2h.wait_stream(stream)
        with torch.cuda.stream(d2h):
            Sh.copy_(Sd.detach(), non_blocking=True)
        Sd.record_stream(d2h)
        stream.wait_stream(h2d)
        Sd.backward(dSd)
        dAh.copy_(Ad.grad, non_blocking=True)
        dBh.copy_(Bd.grad, non_blocking=True)
        stream.wait_stream(d2h)

    for _ in range(2):
        e2e_once()
    torch.cuda.synchronize()
    times = []
    for _ in range(max(3, min(args.steps, 10))):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        e2e_once()
        b.record(stream)
        b.synchronize()
        times.append(a.elapsed_time(b))
    e2e_ms = statistics.mean(times)
    e2e = {"value": round(6.0 * n * M * D / (e2e_ms * 1e-3) / 1e9, 2), "unit": UNIT,
           "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": 4 * (n * D + M * D + n * M),
           "d2h_bytes_per_step": 4 * (n * M + n * D + M * D),
           "api": "cases.cosine_sim.op.candidate + autograd"}

    cpu = None
    if not args.no_cpu_baseline:
        from oracle import reference_port
        threads = os.cpu_count() or 1
        sec, done = reference_port.cos_time_sample(n, M, D, eps, 512, threads,
                                                   min_seconds=0.75 * args.cpu_seconds)
        cpu = {"value": round(6.0 * done * M * D / sec / 1e9, 3), "unit": UNIT, "cores": threads,
               "kind": "port", "sample": f"{done} rows of A (512 per pass) x all {M} rows of B, "
                                         f"fwd+bwd ({sec:.1f} s on {threads} threads)"}
    print(json.dumps({
        "case": "cosine_sim", "metric": metric, "value": round(gflops, 2), "unit": UNIT,
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded A, B, dS ~ N(0,1))",
        "config": {"workload": workload_name, "N": n, "M": M, "D": D,
                   "l2": "flushed before every timed step (256 MiB write + 256 MiB read, outside events)"},
        "ms_fwd": round(ms_fwd, 5), "ms_bwd": round(ms_bwd, 5),
        "pct_roofline_step": round(100.0 * t_roof / (ms * 1e-3), 2),
        "roofline_step_us": round(t_roof * 1e6, 2), "roofline": roofline,
        "gpu_launches": int(launches_per_step * args.steps), "clocks": clocks, "e2e": e2e,
        "cpu_baseline": cpu}), flush=True)
    del step_graph, fwd_graph, bwd_graph


def run_e2e(X, Y, G, g, world, dev, args, shard, op, route=None):
    """Same metric through the public API, host buffers in and out: per step the H2D copy of
    X (this rank's rows), Y and G from pinned memory, forward + backward, and the D2H copy of
    K, dX and dY into pinned memory, all inside the events.  On one GPU the copies overlap the
    compute the way a user would pipeline them: G (needed only by the backward) is copied on a
    side stream during the forward, and K is copied back on another side stream during the
    backward (H2D and D2H use separate copy engines)."""
    import torch
    Xh = X.cpu().pin_memory()
    Yh = Y.cpu().pin_memory()
    Gh = G.cpu().pin_memory()
    n, D = X.shape
    M = Y.shape[0]
    Kh = torch.empty(n, M, dtype=torch.float32).pin_memory()
    dXh = torch.empty(n, D, dtype=torch.float32).pin_memory()
    dYh = torch.empty(M, D, dtype=torch.float32).pin_memory()
    stream = torch.cuda.current_stream(dev)
    h2d = torch.cuda.Stream(device=dev)
    d2h = torch.cuda.Stream(device=dev)

    def one():
        Xd = Xh.to(dev, non_blocking=True)
        Yd = Yh.to(dev, non_blocking=True)
        if world == 1:
            h2d.wait_stream(stream)  # inside the step's timed region
            with torch.cuda.stream(h2d):
                Gd = Gh.to(dev, non_blocking=True)
            Gd.record_stream(stream)
            Xd.requires_grad_(True)
            Yd.requires_grad_(True)
            K = op.candidate({"X": Xd, "Y": Yd}, {"gamma": g})
            d2h.wait_stream(stream)  # K is complete
            with torch.cuda.stream(d2h):
                Kh.copy_(K.detach(), non_blocking=True)
            K.record_stream(d2h)
            stream.wait_stream(h2d)  # G has arrived
            K.backward(Gd)
            dX, dY = Xd.grad, Yd.grad
            dXh.copy_(dX, non_blocking=True)
            dYh.copy_(dY, non_blocking=True)
            stream.wait_stream(d2h)  # the K copy is inside the timed region
        else:
            Gd = Gh.to(dev, non_blocking=True)
            K, dX, dY = shard.forward_backward_shard(Xd, Yd, Gd, g, route=route)
            Kh.copy_(K.detach(), non_blocking=True)
            dXh.copy_(dX, non_blocking=True)
            dYh.copy_(dY, non_blocking=True)

    for _ in range(max(2, args.warmup)):
        one()
    torch.cuda.synchronize()
    times = []
    for _ in range(max(3, min(args.steps, 10))):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        one()
        b.record(stream)
        b.synchronize()
        times.append(a.elapsed_time(b))
    ms = shard.max_over_ranks(statistics.mean(times), device=dev)
    flop = 6.0 * n * world * M * D
    return {"value": round(flop / (ms * 1e-3) / 1e9, 2), "unit": UNIT, "ms_per_step": round(ms, 4),
            "h2d_bytes_per_step": 4 * (n * D + M * D + n * M),
            "d2h_bytes_per_step": 4 * (n * M + n * D + M * D),
            "api": "cases.rbf.op.candidate + autograd" if world == 1
                   else "cases.rbf.shard.forward_backward_shard"}


if __name__ == "__main__":
    main()
