"""Upstream vLLM (0.22) with the foundry graph extension on one GPU: two
SAVE passes and a fresh LOAD of the engine's own FULL_DECODE_ONLY graphs
(cuBLAS, Inductor/Triton, vLLM and attention kernels, programmatic launch
edges); LOAD must restore every graph and produce SAVE's greedy tokens.
Each pass is a fresh process (foundry_b200.integration.vllm.check)."""

import importlib.util
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(importlib.util.find_spec("vllm") is None, reason="vLLM is not installed")
def test_vllm_save_load_restores_the_engines_graphs(tmp_path):
    env = dict(os.environ, PYTHONPATH=ROOT)
    r = subprocess.run([sys.executable, "-m", "foundry_b200.integration.vllm.check", "--workdir", str(tmp_path),
                        "--sizes", "1,2,4,8", "--gen", "12"], env=env, capture_output=True, text=True, timeout=1500)
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert lines, f"rc {r.returncode}\n{r.stdout[-2000:]}\n{r.stderr[-4000:]}"
    out = json.loads(lines[-1])
    assert out["tokens_match"] and out["save_passes_match"], out
    assert out["graphs_restored"] == out["graphs_saved"] == 4, out
