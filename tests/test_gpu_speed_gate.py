"""The reference harness's speed gate on the B200: framework.bench.compare times the candidate
against torch.compile(reference_forward) on the case's default size (N = M = 2048, D = 64, the
reference's own RBF_SIZE), forward and backward separately, and passes at >= 1.05x on both with
every coefficient of variation within 5% (reference framework/bench.py:129-178 and the --strict
gate of skill/scripts/bench_case.py:82-85)."""
import os
import re

import pytest

pytestmark = pytest.mark.gpu


def _speedups(report):
    f = re.search(r"forward : ([0-9.]+)x", report)
    b = re.search(r"backward: ([0-9.]+)x", report)
    assert f and b, report
    return float(f.group(1)), float(b.group(1))


@pytest.mark.parametrize("case_name", ["rbf", "cosine_sim"])
def test_speed_gate_vs_torch_compile(case_name, cuda_device):
    import importlib
    from framework.bench import compare
    case = importlib.import_module(f"cases.{case_name}").CASE
    candidate = importlib.import_module(f"cases.{case_name}.op").candidate
    report, passed = compare(case, candidate, device="cuda")
    print(report)
    out = os.environ.get("RBF_SPEED_GATE_LOG")
    if out:
        with open(out, "a") as f:
            f.write(report + "\n\n")
    fwd, bwd = _speedups(report)
    assert fwd >= 1.05 and bwd >= 1.05, report
    # The gate's verdict also needs every CV in bounds; a noisy host may void a measurement
    # (the harness then asks for a re-run), which is not a failure of the candidate.
    assert passed or "CV over threshold" in report, report
