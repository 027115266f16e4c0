"""Tensor-parallel serving (>= 2 GPUs): every rank holds a shard of the same
full weights; prefill and decode (eager and graph-replayed) must give the
fp32 reference's greedy tokens on every rank, and a SAVEd TP archive must
LOAD in fresh processes and replay to the same tokens. Ranks are child
processes; gloo bootstraps, every collective is our own kernel over
symmetric memory."""

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
import json, os, sys, types
sys.path.insert(0, ROOT)
import torch, torch.distributed as dist
torch.cuda.set_device(RANK)
dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % PORT, rank=RANK, world_size=WORLD)
from foundry_b200 import ops
from foundry_b200.models.llama import tiny, reference_forward
from foundry_b200.runner.engine import EngineConfig, LLMEngine
from foundry_b200.runner import persist

cfg = tiny(layers=2, vocab=4096)

def full_weights():
    g = torch.Generator(device="cuda").manual_seed(1234)
    h, d = cfg.hidden, cfg.head_dim
    rnd = lambda std, *s: (torch.randn(*s, device="cuda", generator=g) * std).to(torch.bfloat16)
    nrm = lambda n: (1 + 0.1 * torch.randn(n, device="cuda", generator=g)).to(torch.bfloat16)
    full = {"embed": rnd(1.0, cfg.vocab, h)}
    for i in range(cfg.layers):
        full[f"layers.{i}.attn_norm"] = nrm(h)
        full[f"layers.{i}.qkv"] = rnd(0.02, cfg.qkv_dim, h)
        full[f"layers.{i}.o"] = rnd(0.02, h, cfg.n_q * d)
        full[f"layers.{i}.mlp_norm"] = nrm(h)
        full[f"layers.{i}.gate_up"] = rnd(0.02, 2 * cfg.inter, h)
        full[f"layers.{i}.down"] = rnd(0.02, h, cfg.inter)
    full["final_norm"] = nrm(h)
    full["lm_head"] = rnd(0.1, cfg.vocab, h)
    return full

def as_model(full):
    m = types.SimpleNamespace(embed=full["embed"], final_norm=full["final_norm"], lm_head=full["lm_head"])
    m.layers = [{k: full[f"layers.{i}.{k}"] for k in ("attn_norm", "qkv", "o", "mlp_norm", "gate_up", "down")}
                for i in range(cfg.layers)]
    return m

g = torch.Generator().manual_seed(5)
PROMPTS = [torch.randint(0, cfg.vocab, (n,), generator=g).tolist() for n in (3, 17, 64, 65, 100)]
GEN = 8

def same_on_all_ranks(obj):
    got = [None] * WORLD
    dist.all_gather_object(got, obj)
    assert all(o == got[0] for o in got), got

def check_images():
    for img in ("comm", "gemm_bf16", "elementwise", "attention_tc"):
        assert ops.status(img) == 0, (img, ops.status(img))
"""

SAVE = COMMON + r"""
ecfg = EngineConfig(model=cfg, max_batch=16, max_seq_len=256, max_prefill_tokens=512, max_prefill_seqs=8,
                    graph_sizes=[1, 2, 4, 8, 16], region_base=0x620000000000, region_size="8GB", tp=WORLD)
eng = LLMEngine(ecfg, init_weights=False)
assert eng.weights.nq_l == cfg.n_q // WORLD and eng.state.logits.shape[1] == cfg.vocab // WORLD
full = full_weights()
eng.weights.load_full(full)
out_eager = eng.generate(PROMPTS, GEN)
same_on_all_ranks(out_eager)
# greedy tokens against the fp32 reference (skip near-ties)
ref_w = as_model(full)
checked = 0
for p, o in zip(PROMPTS, out_eager):
    seq = p + o[:-1]
    logits = reference_forward(cfg, ref_w, torch.tensor(seq, device="cuda"), eng.cos_sin)
    for j in range(GEN):
        top2 = logits[len(p) - 1 + j].topk(2)
        if top2.values[0] - top2.values[1] > 0.25:
            assert o[j] == int(top2.indices[0]), (p[:4], j, o, top2)
            checked += 1
assert checked >= len(PROMPTS) * GEN // 2, checked
persist.save(eng, ARCHIVE)  # captures the decode graphs
out_graph = eng.generate(PROMPTS, GEN)
assert out_graph == out_eager, (out_graph, out_eager)
check_images()
if RANK == 0:
    with open(os.path.join(ARCHIVE, "tokens.json"), "w") as f:
        json.dump(out_eager, f)
dist.barrier()
eng.close()
dist.destroy_process_group()
print("RANK_OK", RANK, "checked", checked, "multicast", eng.tp is None)
"""

LOAD = COMMON + r"""
eng, t = persist.load(ARCHIVE, init_weights=False)
eng.weights.load_full(full_weights())
assert len(eng.graphs) == 5
out = eng.generate(PROMPTS, GEN)
with open(os.path.join(ARCHIVE, "tokens.json")) as f:
    want = json.load(f)
assert out == want, (out, want)
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


def _run_ranks(body, world, archive, reduce="nvls"):
    port = _free_port()
    # FOUNDRY_TP_REDUCE=nvls: prefill rows (>= 128) take the NVLS reduce path
    # even at 2 ranks, decode rows the multicast slot exchange; "fused": every
    # row-parallel GEMM all-reduces in its own epilogue
    env = dict(os.environ, PYTHONPATH=ROOT, NCCL_NVLS_ENABLE="0", FOUNDRY_TP_REDUCE=reduce)
    procs = []
    for rank in range(world):
        code = f"ROOT={ROOT!r}; PORT={port}; RANK={rank}; WORLD={world}; ARCHIVE={archive!r}\n" + body
        procs.append(subprocess.Popen([sys.executable, "-c", code], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.PIPE, text=True))
    outs = [p.communicate(timeout=900) for p in procs]
    for p, (o, e) in zip(procs, outs):
        assert p.returncode == 0, f"{o[-2000:]}\n{e[-6000:]}"
        assert "RANK_OK" in o


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs >= 2 GPUs")
def test_tensor_parallel_decode_save_load(tmp_path):
    world = 2 if torch.cuda.device_count() < 4 else min(torch.cuda.device_count(), 8)
    archive = str(tmp_path / "tp_archive")
    _run_ranks(SAVE, world, archive)
    _run_ranks(LOAD, world, archive)


AR_KERNEL = r"""
import os, sys
sys.path.insert(0, ROOT)
import torch, torch.distributed as dist
torch.cuda.set_device(RANK)
dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % PORT, rank=RANK, world_size=WORLD)
from foundry_b200 import ops
from foundry_b200.ops import _rt
from foundry_b200.runner.engine import TPContext
from foundry_b200.graphs import CUDAGraph, graph

ROWS, H = 1024, 1024
tp = TPContext(ROWS, H, 16)
ex = tp.slots
assert ex.symm.multicast, "no NVLS multicast on this node"
g = torch.Generator(device="cuda").manual_seed(99)
for t, k in ((7, 512), (64, 2048), (256, 1024), (300, 512), (1024, 256)):
    # every rank's own x and w shard; the reference sums all ranks' products
    xs = [(torch.randn(t, k, device="cuda", generator=g) * 0.5).to(torch.bfloat16) for _ in range(WORLD)]
    ws = [(torch.randn(H, k, device="cuda", generator=g) * 0.05).to(torch.bfloat16) for _ in range(WORLD)]
    ref = sum(x.float() @ w.float().T for x, w in zip(xs, ws))
    for which in (0, 1, 0, 1):  # parity of each control block flips every launch
        ex.slot(which, 1)[:t].fill_(float("nan"))
        dist.barrier()
        with _rt.pdl():
            assert ex.gemm_allreduce(xs[RANK], ws[RANK], which)
        torch.cuda.synchronize()
        got = ex.slot(which, 1)[:t].float()
        torch.testing.assert_close(got, ref, atol=3e-2, rtol=2e-2)
        dist.barrier()
    # captured in a CUDA graph and replayed (the epoch advances on the device)
    gr = CUDAGraph()
    with graph(gr):
        with _rt.pdl():
            ex.gemm_allreduce(xs[RANK], ws[RANK], 0)
            ex.gemm_allreduce(xs[RANK], ws[RANK], 1)
    for _ in range(3):
        ex.slot(0, 1)[:t].zero_()
        ex.slot(1, 1)[:t].zero_()
        dist.barrier()
        gr.replay()
        torch.cuda.synchronize()
        torch.testing.assert_close(ex.slot(0, 1)[:t].float(), ref, atol=3e-2, rtol=2e-2)
        torch.testing.assert_close(ex.slot(1, 1)[:t].float(), ref, atol=3e-2, rtol=2e-2)
        dist.barrier()
    del gr
assert ops.status("gemm_bf16") == 0, ops.status("gemm_bf16")
dist.barrier()
tp.close()
dist.destroy_process_group()
print("RANK_OK", RANK)
"""


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs >= 2 GPUs")
def test_fused_gemm_allreduce_kernel():
    """fb_gemm_bf16_ar_bn*: the row-parallel GEMM whose epilogue all-reduces
    its tiles over NVSwitch equals the fp32 sum of every rank's product, on
    swap-AB (decode) and token-major (prefill) shapes, on repeated launches
    of both control blocks and replayed from a CUDA graph."""
    world = min(torch.cuda.device_count(), 8)
    _run_ranks(AR_KERNEL, world, "")


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs >= 2 GPUs")
def test_tensor_parallel_fused_allreduce_save_load(tmp_path):
    """The TP engine with every row-parallel GEMM all-reducing in its own
    epilogue: greedy tokens match the fp32 reference, and a SAVEd archive
    LOADs and replays to the same tokens."""
    world = 2 if torch.cuda.device_count() < 4 else min(torch.cuda.device_count(), 8)
    archive = str(tmp_path / "tp_fused_archive")
    _run_ranks(SAVE, world, archive, reduce="fused")
    _run_ranks(LOAD, world, archive, reduce="fused")
