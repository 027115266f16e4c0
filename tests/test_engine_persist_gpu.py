"""Single-GPU engine SAVE -> LOAD in fresh processes: the restored decode
graphs reproduce the SAVE process's greedy tokens; after the first decode
step every restored graph gets its own executable on a background thread,
and a second generation through those executables gives the same tokens."""

import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

COMMON = r"""
import json, os, sys
sys.path.insert(0, ROOT)
import torch
from foundry_b200 import ops
from foundry_b200.models.llama import tiny
from foundry_b200.runner.engine import EngineConfig, LLMEngine
from foundry_b200.runner import persist

cfg = tiny(layers=2, vocab=4096)
g = torch.Generator().manual_seed(3)
PROMPTS = [torch.randint(0, cfg.vocab, (n,), generator=g).tolist() for n in (5, 40, 64, 100, 17)]
"""

SAVE = COMMON + r"""
ecfg = EngineConfig(model=cfg, max_batch=8, max_seq_len=256, max_prefill_tokens=512, max_prefill_seqs=8,
                    graph_sizes=[1, 2, 4, 8], region_base=0x640000000000, region_size="8GB")
eng = LLMEngine(ecfg)
persist.save(eng, ARCHIVE)
out = eng.generate(PROMPTS, 12)
json.dump(out, open(os.path.join(ARCHIVE, "tokens.json"), "w"))
eng.close()
print("SAVE_OK")
"""

LOAD = COMMON + r"""
eng, t = persist.load(ARCHIVE)
assert len(eng.graphs) == 4 and eng.materialize_after_first_step
want = json.load(open(os.path.join(ARCHIVE, "tokens.json")))
out = eng.generate(PROMPTS, 12)
assert out == want, (out, want)
eng.wait_materialized()
assert all(g._restored.materialized for g in eng.graphs.values())
out2 = eng.generate(PROMPTS, 12)
assert out2 == want, (out2, want)
for img in ("gemm_bf16", "elementwise", "attention_tc"):
    assert ops.status(img) == 0, img
eng.close()
print("LOAD_OK", t["num_graphs"], t["num_groups"])
"""


def _run(body, archive):
    env = dict(os.environ, PYTHONPATH=ROOT)
    code = f"ROOT={ROOT!r}; ARCHIVE={archive!r}\n" + body
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    return r.stdout


def test_engine_save_load_and_background_materialize(tmp_path):
    archive = str(tmp_path / "arch")
    assert "SAVE_OK" in _run(SAVE, archive)
    out = _run(LOAD, archive)
    assert "LOAD_OK 4" in out, out
