"""bench.py contract pieces that need no GPU: the reference arm prints one
JSON line with ``impl`` and ``unavailable`` and exits 0; model presets fill
the workload of each named config; explicit flags override them."""

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_reports_unavailable():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--gpus", "1",
                        "--steps", "3", "--warmup", "3"], capture_output=True, text=True, timeout=120, cwd="/")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    out = json.loads(lines[0])
    assert out["impl"] == "reference" and out["unavailable"]


@pytest.mark.parametrize("argv,want", [
    ([], {"model": "llama-3-8b", "batch": 256, "prompt_len": 512, "parallel": "dp", "steps": 50, "warmup": 5}),
    (["--model", "qwen3-30b-a3b"], {"batch": 512, "prompt_len": 1024, "parallel": "ep", "graph_sizes": "2:512:2"}),
    (["--model", "llama-3-70b"], {"batch": 1024, "prompt_len": 2048, "parallel": "tp"}),
    (["--model", "llama-3-8b", "--batch", "64", "--steps", "7"], {"batch": 64, "steps": 7, "prompt_len": 512}),
])
def test_presets(monkeypatch, argv, want):
    sys.path.insert(0, ROOT)
    import bench

    monkeypatch.setattr(sys, "argv", ["bench.py", *argv])
    args = bench.parse()
    for k, v in want.items():
        assert getattr(args, k) == v, (k, getattr(args, k), v)


def test_replica_visibility():
    """A data-parallel replica's child processes see only their own GPU."""
    import bench

    assert bench.replica_visibility(3, {}) == ({"CUDA_VISIBLE_DEVICES": "3"}, 0)
    assert bench.replica_visibility(1, {"CUDA_VISIBLE_DEVICES": "4,5,6"}) == ({"CUDA_VISIBLE_DEVICES": "5"}, 0)
    assert bench.replica_visibility(0, {"CUDA_VISIBLE_DEVICES": "GPU-abc, GPU-def"}) == (
        {"CUDA_VISIBLE_DEVICES": "GPU-abc"}, 0)
    assert bench.replica_visibility(2, {"CUDA_VISIBLE_DEVICES": ""}) == ({"CUDA_VISIBLE_DEVICES": "2"}, 0)
