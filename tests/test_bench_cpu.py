"""The bench.py contract on a machine without a GPU: the reference arm answers with
one JSON line (its result or why it is unavailable) and exits 0, and the CPU
workload (config 1) prints one well-formed JSON line."""
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _run(*args, timeout=900):
    env = dict(os.environ, PYTHONPATH=str(ROOT))
    env.pop("CUDA_VISIBLE_DEVICES", None)
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, env=env, capture_output=True,
                          text=True, timeout=timeout)


def _json_lines(text):
    return [json.loads(x) for x in text.splitlines() if x.startswith("{")]


def test_reference_arm_prints_one_line_and_exits_zero():
    res = _run("--impl", "reference", "--gpus", "1", "--steps", "3", "--warmup", "3")
    assert res.returncode == 0, res.stderr[-2000:]
    lines = _json_lines(res.stdout)
    assert len(lines) == 1 and lines[0]["impl"] == "reference"
    assert "unavailable" in lines[0] or lines[0].get("value", 0) > 0


def test_cpu_workload_line():
    res = _run("--workload", "tgn_cpu", "--steps", "3", "--warmup", "3")
    assert res.returncode == 0, res.stderr[-2000:]
    lines = _json_lines(res.stdout)
    assert len(lines) == 1
    line = lines[0]
    for key in ("metric", "value", "unit", "steps", "warmup", "ms_per_step", "higher_is_better", "dtype", "data",
                "config"):
        assert key in line, key
    assert line["value"] > 0 and line["steps"] == 3 and line["warmup"] == 3 and line["dtype"] == "fp32"
    assert line["config"]["events"] == 157474 and line["config"]["global_batch"] == 200


def test_gpu_workload_without_a_gpu_says_so():
    import pytest
    import torch

    if torch.cuda.is_available():
        pytest.skip("a CUDA device is visible: the GPU workload would run")
    res = _run("--steps", "3", "--warmup", "3", timeout=300)
    assert res.returncode == 2 and "CUDA" in res.stderr and "Traceback" not in res.stderr
