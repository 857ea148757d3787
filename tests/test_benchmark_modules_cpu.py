"""Every benchmark driver imports and parses its arguments without a GPU
(`python -m multi_gpu_flashattention_b200.benchmarks.<name> --help`), so a
broken import or parser in a GPU-only driver shows up on the host."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
MODULES = ["profile_kernels", "ring_trace", "ring_train",
           "single_gpu_baseline", "single_gpu_shapes", "ring_attention", "ring_loop",
           "ring_oneshot", "layout_balance", "check_peer", "probes", "reference_programs",
           "fwd_tuning"]


@pytest.mark.parametrize("name", MODULES)
def test_driver_help(name):
    p = subprocess.run([sys.executable, "-m", f"multi_gpu_flashattention_b200.benchmarks.{name}",
                        "--help"], cwd=ROOT, capture_output=True, text=True, timeout=180)
    assert p.returncode == 0, p.stderr[-2000:]
    assert "usage:" in p.stdout


def test_every_driver_is_listed():
    here = os.path.join(ROOT, "multi_gpu_flashattention_b200", "benchmarks")
    found = {f[:-3] for f in os.listdir(here)
             if f.endswith(".py") and f not in ("__init__.py", "common.py")}
    assert found == set(MODULES), found ^ set(MODULES)


@pytest.mark.parametrize("script", ["train_ring_lm.py", "ring_attention_quickstart.py"])
def test_example_help(script):
    p = subprocess.run([sys.executable, os.path.join(ROOT, "examples", script), "--help"],
                       cwd=ROOT, capture_output=True, text=True, timeout=180)
    assert p.returncode == 0 and "usage:" in p.stdout, p.stderr[-2000:]
