"""The LD_PRELOAD interposer on the real driver: region placement of torch
allocations, stop/resume, preallocation, a torch graph (cuBLAS GEMMs +
elementwise kernels from libtorch) saved in one process and restored in
another, bit-exact, and 12 such graphs restored asynchronously."""

import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
HOOK = os.path.join(ROOT, "foundry_b200", "lib", "libfoundry_hook.so")


def _run(name, workdir, timeout=300):
    env = dict(os.environ, LD_PRELOAD=HOOK, PYTHONPATH=ROOT, TORCH_CUBLASLT_UNIFIED_WORKSPACE="1")
    res = subprocess.run([sys.executable, os.path.join(HERE, "interposer_scenarios.py"), name, workdir], env=env,
                         capture_output=True, text=True, timeout=timeout)
    assert res.returncode == 0, f"{name} failed:\n{res.stdout[-3000:]}\n{res.stderr[-5000:]}"
    return json.loads(res.stdout.strip().splitlines()[-1])


def test_region_allocations(tmp_path):
    assert _run("region", str(tmp_path))["ok"]


def test_preallocation(tmp_path):
    assert _run("prealloc", str(tmp_path))["ok"]


def test_torch_graph_save_load(tmp_path):
    info = _run("graph_save", str(tmp_path))
    assert info["nodes"] > 2
    assert _run("graph_load", str(tmp_path))["ok"]


def test_async_restore_of_graphs_sharing_topologies(tmp_path):
    """12 graphs at batch sizes 8..1024 with repeats (members share topology
    templates), restored with start_graph_builds overlapped with host work."""
    info = _run("async_save", str(tmp_path))
    assert info["graphs"] == 12 and info["groups"] < 12, info
    assert _run("async_load", str(tmp_path))["ok"]


def test_random_numbers_in_a_restored_graph(tmp_path):
    """torch.rand and dropout inside a captured graph: the restored graph,
    replayed from the same seed, draws the same numbers as the SAVE process's
    replays (the generator's seed/offset words are relocated and rewritten
    before each replay)."""
    info = _run("rng_save", str(tmp_path))
    assert info["increment"] > 0
    assert _run("rng_load", str(tmp_path))["ok"]


def test_torch_compile_graph_save_load(tmp_path):
    """A torch.compile'd function (Inductor fuses it into a Triton kernel) is
    captured and saved; a fresh process that compiles nothing restores it
    from the archive's packed image and replays it bit-exact."""
    info = _run("compile_save", str(tmp_path), timeout=600)
    assert info["adopted"] >= 1
    assert _run("compile_load", str(tmp_path))["ok"]
