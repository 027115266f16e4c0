"""Expert parallelism with DP attention (>= 2 GPUs): Qwen3-MoE shapes, each
rank serving its own prompts while the experts are sharded. The fused
quantise+dispatch and GEMM+combine exchange must reproduce the single-GPU
engine's tokens exactly (the per-token math is the same, only the rows move),
eagerly and from captured graphs, and a SAVEd EP archive must LOAD in fresh
processes and replay to the same tokens."""

import json
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

COMMON = r"""
import json, os, sys
sys.path.insert(0, ROOT)
import torch
torch.cuda.set_device(RANK)
from foundry_b200 import ops
from foundry_b200.models.qwen3_moe import tiny_moe
from foundry_b200.runner.engine import EngineConfig, LLMEngine
from foundry_b200.runner import persist

cfg = tiny_moe(layers=2, vocab=4096, experts=32)
g = torch.Generator().manual_seed(11)
PROMPTS = {r: [torch.randint(0, cfg.vocab, (n,), generator=g).tolist() for n in (4, 33, 70, 129, 9)]
           for r in range(8)}
GEN = 6

def ecfg(ep, base):
    return EngineConfig(model=cfg, max_batch=16, max_seq_len=256, max_prefill_tokens=512, max_prefill_seqs=8,
                        graph_sizes=[1, 2, 4, 8, 16], region_base=base, region_size="8GB", ep=ep)

def check_images():
    for img in ("comm", "moe", "gemm_bf16", "elementwise", "attention_tc"):
        assert ops.status(img) == 0, (img, ops.status(img))
"""

REFERENCE = COMMON + r"""
eng = LLMEngine(ecfg(1, None))
out = {r: eng.generate(PROMPTS[r], GEN) for r in range(WORLD)}
check_images()
with open(os.path.join(ARCHIVE, "reference.json"), "w") as f:
    json.dump(out, f)
print("RANK_OK ref")
"""

SAVE = COMMON + r"""
import torch.distributed as dist
dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % PORT, rank=RANK, world_size=WORLD)
with open(os.path.join(ARCHIVE, "reference.json")) as f:
    want = json.load(f)[str(RANK)]
eng = LLMEngine(ecfg(WORLD, 0x640000000000))
assert eng.weights.e_local == cfg.num_experts // WORLD
eager = eng.generate(PROMPTS[RANK], GEN)
assert eager == want, (RANK, eager, want)
persist.save(eng, ARCHIVE)
graph = eng.generate(PROMPTS[RANK], GEN)
assert graph == want, (RANK, graph, want)
check_images()
dist.barrier()
eng.close()
dist.destroy_process_group()
print("RANK_OK", RANK)
"""

LOAD = COMMON + r"""
import torch.distributed as dist
dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % PORT, rank=RANK, world_size=WORLD)
with open(os.path.join(ARCHIVE, "reference.json")) as f:
    want = json.load(f)[str(RANK)]
eng, t = persist.load(ARCHIVE)
assert len(eng.graphs) == 5
out = eng.generate(PROMPTS[RANK], GEN)
assert out == want, (RANK, out, want)
check_images()
dist.barrier()
eng.close()
dist.destroy_process_group()
print("RANK_OK", RANK, "restore_s", t["restore_s"])
"""


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _run(body, ranks, world, archive):
    port = _free_port()
    env = dict(os.environ, PYTHONPATH=ROOT, NCCL_NVLS_ENABLE="0")
    procs = []
    for rank in ranks:
        code = f"ROOT={ROOT!r}; PORT={port}; RANK={rank}; WORLD={world}; ARCHIVE={archive!r}\n" + body
        procs.append(subprocess.Popen([sys.executable, "-c", code], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.PIPE, text=True))
    outs = [p.communicate(timeout=900) for p in procs]
    bad = [f"--- rank {r} rc={p.returncode}\n{o[-1500:]}\n{e[-3000:]}" for r, p, (o, e) in zip(ranks, procs, outs)
           if p.returncode != 0 or "RANK_OK" not in o]
    assert not bad, "\n".join(bad)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs >= 2 GPUs")
def test_expert_parallel_matches_single_gpu_and_restores(tmp_path):
    world = 2 if torch.cuda.device_count() < 4 else min(torch.cuda.device_count(), 8)
    archive = str(tmp_path / "ep_archive")
    os.makedirs(archive)
    _run(REFERENCE, [0], world, archive)
    _run(SAVE, range(world), world, archive)
    _run(LOAD, range(world), world, archive)
