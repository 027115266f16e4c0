"""Multi-GPU (>= 2): symmetric memory at identical addresses, the flag barrier,
one-shot and NVLS all-reduce, the fused GEMM -> multicast slots -> add+RMSNorm
all-reduce, and the vocab-sharded argmax. Each rank is a child process
(gloo for the bootstrap, our own kernels for every collective)."""

import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

WORKER = r"""
import os, sys, math
sys.path.insert(0, ROOT)
import torch, torch.distributed as dist
torch.cuda.set_device(RANK)
dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % PORT, rank=RANK, world_size=WORLD)
from foundry_b200 import ops
from foundry_b200.parallel.symm import SymmetricMemory, CTRL_BYTES
from foundry_b200.parallel import comm
from foundry_b200.graphs import tensor_from_ptr

s = SymmetricMemory(256 << 20)
W, R = s.world, s.rank
# 1) peer visibility through the flag barrier (peer memory is read by our
#    kernels over P2P; torch cannot wrap another device's memory)
n = 4096
mine = s.tensor(R, (n,), torch.bfloat16, CTRL_BYTES)
mine.fill_(float(R + 1))
tot = torch.empty(n, dtype=torch.bfloat16, device="cuda")
comm.all_reduce(s, CTRL_BYTES, n, tot)
assert torch.all(tot == float(W * (W + 1) // 2)), tot[:4]
comm.barrier(s)
# 2) all-reduce, one-shot (deterministic) and NVLS
g = torch.Generator(device="cuda").manual_seed(100 + R)
x = torch.randn(1 << 20, device="cuda", generator=g).to(torch.bfloat16)
off = CTRL_BYTES + (1 << 20)
s.tensor(R, x.shape, torch.bfloat16, off).copy_(x)
allx = [torch.randn(1 << 20, device="cuda", generator=torch.Generator(device="cuda").manual_seed(100 + r)).to(torch.bfloat16) for r in range(W)]
ref = sum(t.float() for t in allx)
out = torch.empty_like(x)
comm.all_reduce(s, off, x.numel(), out, algo="oneshot")
torch.testing.assert_close(out.float(), ref, atol=3e-2 * W, rtol=2e-2)
comm.barrier(s)
if s.multicast:
    out2 = torch.empty_like(x)
    comm.all_reduce(s, off, x.numel(), out2, algo="nvls")
    torch.testing.assert_close(out2.float(), ref, atol=3e-2 * W, rtol=2e-2)
    comm.barrier(s)
# 3) fused GEMM -> multicast slots -> add + RMSNorm (row-parallel layer);
#    T = 64 runs the swap-AB (transposed) epilogue, T = 320 the row-major one
for which, T in ((0, 64), (1, 320)):
    H, Kr = 1024, 512
    ex = comm.SlotExchange(s, CTRL_BYTES + (16 << 20), 320, H)
    gw = torch.Generator(device="cuda").manual_seed(7 + T)
    xs = [torch.randn(T, Kr, device="cuda", generator=gw).to(torch.bfloat16) for _ in range(W)]
    ws = [(torch.randn(H, Kr, device="cuda", generator=gw) * 0.05).to(torch.bfloat16) for _ in range(W)]
    h0 = torch.randn(T, H, device="cuda", generator=gw).to(torch.bfloat16)
    nw = torch.randn(H, device="cuda", generator=gw).to(torch.bfloat16)
    tgt = ex.gemm_target(which)
    if tgt:
        ops.linear_multicast(xs[R], ws[R], tgt)
    else:
        ops.linear(xs[R], ws[R], out=ex.local_slot(which)[:T])
        ex.broadcast_local_slot(which, T)
    comm.barrier(s)
    h = h0.clone(); xo = torch.empty_like(h)
    comm.add_rmsnorm_slots(ex.local_slots(which), T, h, nw, xo, 1e-5)
    part = [(xs[r].float() @ ws[r].float().T).to(torch.bfloat16).float() for r in range(W)]
    href = (sum(part) + h0.float())
    torch.testing.assert_close(h.float(), href, atol=6e-2, rtol=2e-2)
    hf = h.float()
    torch.testing.assert_close(xo.float(), hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-5) * nw.float(), atol=3e-2, rtol=2e-2)
    comm.barrier(s)
# 4) vocab-sharded greedy argmax
V = 4000
full = torch.randn(T, V * W, device="cuda", generator=torch.Generator(device="cuda").manual_seed(9)).to(torch.bfloat16)
ids = torch.empty(T, dtype=torch.int32, device="cuda")
comm.argmax_sharded(s, full[:, R * V:(R + 1) * V].contiguous(), R * V, CTRL_BYTES + (128 << 20), ids)
assert torch.equal(ids.long(), full.float().argmax(-1)), (ids[:8], full.float().argmax(-1)[:8])
for img in ("comm", "gemm_bf16"):
    assert ops.status(img) == 0, img
comm.barrier(s)
torch.cuda.synchronize()
dist.barrier()
s.close()
dist.destroy_process_group()
print("RANK_OK", R, "multicast", s.multicast)
"""


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs >= 2 GPUs")
def test_symmetric_collectives_and_fused_gemm_allreduce():
    world = min(torch.cuda.device_count(), 8)
    port = _free_port()
    env = dict(os.environ, PYTHONPATH=ROOT, NCCL_NVLS_ENABLE="0")
    procs = []
    for rank in range(world):
        code = f"ROOT={ROOT!r}; PORT={port}; RANK={rank}; WORLD={world}\n" + WORKER
        procs.append(subprocess.Popen([sys.executable, "-c", code], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.PIPE, text=True))
    outs = [p.communicate(timeout=600) for p in procs]
    for p, (o, e) in zip(procs, outs):
        assert p.returncode == 0, f"{o[-2000:]}\n{e[-4000:]}"
        assert "RANK_OK" in o
