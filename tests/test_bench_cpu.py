"""bench.py's reference arm runs on the host cores (no GPU): its JSON line keeps the bench
contract for both cases, and a non-zero rank under torchrun prints nothing and exits 0."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(args, env_extra=None):
    env = dict(os.environ, **(env_extra or {}))
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py")] + args, cwd=ROOT,
                       capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stdout + r.stderr
    return [json.loads(ln) for ln in r.stdout.splitlines() if ln.startswith("{")]


@pytest.mark.parametrize("case_args", [[], ["--case", "cosine_sim", "--cpu-seconds", "2"]])
def test_reference_arm_json_line(case_args):
    lines = _run(["--impl", "reference", "--steps", "1", "--warmup", "0"] + case_args)
    assert len(lines) == 1
    d = lines[0]
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["value"] > 0 and d["unit"] == "GFLOP/s" and d["higher_is_better"] is True
    assert d["steps"] == 1 and d["warmup"] == 0 and d["n_gpus"] == 1
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    assert d["config"]["N"] == d["config"]["M"] == 4096 and d["config"]["D"] == 64


def test_reference_arm_other_ranks_do_no_work():
    lines = _run(["--impl", "reference", "--steps", "1", "--warmup", "0"],
                 {"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"})
    assert lines == []
