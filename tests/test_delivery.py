"""The standalone C++ delivery harness (cases/rbf/delivery): builds against the library on CPU;
on a GPU it must print PASS through both ABIs."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DELIVERY = os.path.join(ROOT, "nl2cuda-kernel-agent_b200", "cases", "rbf", "delivery")


def build(out_dir):
    if shutil.which("g++") is None:
        pytest.skip("no C++ compiler")
    r = subprocess.run(["make", f"OUT={out_dir}"], cwd=DELIVERY, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    exe = os.path.join(out_dir, "rbf_selftest")
    assert os.access(exe, os.X_OK)
    return exe


def test_delivery_harness_builds(tmp_path):
    build(str(tmp_path))


@pytest.mark.gpu
@pytest.mark.parametrize("args", [[], ["200", "300", "48", "0.02", "7"], ["129", "260", "100", "0.01", "3"]])
def test_delivery_harness_passes(tmp_path, args, cuda_device):
    exe = build(str(tmp_path))
    r = subprocess.run([exe] + args, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and "PASS" in r.stdout, r.stdout + r.stderr
