"""Device-timed roofline report of the fused compute + collective paths
(run under torchrun, one rank per GPU; every number is the max over ranks).

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
        -m foundry_b200.runner.profile_comm [--reps 20]

Paths:
  tp_slots   row-parallel GEMM whose epilogue multicasts each tile into every
             rank's slot (multimem.st), flag barrier, rank-ordered add +
             RMSNorm (Llama-3-70B down projection shapes, tp = N)
  tp_nvls    same GEMM into the local slot, barrier, NVLS reduce-scatter +
             multicast (multimem.ld_reduce / multimem.st), barrier, add + RMSNorm
  gemm_ar    one kernel: the GEMM epilogue reduces each tile in the switch
             once every rank has it and multicasts the sums, then add + RMSNorm
  ep         Qwen3-30B-A3B MoE layer exchange at 512 tokens per rank: count
             exchange + plan + fused e4m3 quantise/dispatch (P2P stores),
             grouped GEMMs, down GEMM with the combine fused into its epilogue

Roofline of a path: the slowest of its FLOPs at the measured sustained bf16
(or 2x for e4m3) tensor rate, its HBM bytes at the measured copy bandwidth,
and the bytes that must cross NVLink per rank at 770 GB/s per direction.
Each segment is timed as a CUDA graph of ``reps`` back-to-back repetitions.
"""

from __future__ import annotations

import argparse
import json
import math
import os

import torch
import torch.distributed as dist

HBM = 6543e9
BF16 = 1369.6e12
NVLINK = 770e9


def _peaks():
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                     "MEASURED_PEAKS.json")
    global HBM, BF16
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        HBM = d.get("hbm_gbs", 6543.1) * 1e9
        BF16 = d.get("bf16_tflops_sustained", 1369.6) * 1e12


def graph_time_us(fn, reps: int) -> float:
    fn()
    torch.cuda.synchronize()
    dist.barrier()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.graph(g, stream=s):
        for _ in range(reps):
            fn()
    g.replay()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) * 1e3 / reps], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    del g
    return float(t.item())


def tp_paths(reps: int) -> dict:
    from .. import ops
    from ..parallel import comm
    from ..parallel.symm import CTRL_BYTES, SymmetricMemory

    w_ = dist.get_world_size()
    hidden, inter = 8192, 28672
    k = inter // w_
    out = {}
    ar_off = -(-(CTRL_BYTES + 2 * w_ * 1024 * hidden * 2) // 4096) * 4096
    symm = SymmetricMemory(ar_off + 2 * comm.AR_BLOCK_BYTES + (1 << 20))
    ex = comm.SlotExchange(symm, CTRL_BYTES, 1024, hidden, ar_offset=ar_off)
    symm.tensor(symm.rank, (2 * comm.AR_BLOCK_BYTES,), torch.uint8, ar_off).zero_()
    torch.cuda.synchronize()
    dist.barrier()
    g = torch.Generator(device="cuda").manual_seed(1 + symm.rank)
    wt = (torch.randn(hidden, k, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    nw = torch.ones(hidden, dtype=torch.bfloat16, device="cuda")
    for b in (64, 256, 1024):
        x = torch.randn(b, k, device="cuda", generator=g).to(torch.bfloat16)
        h = torch.zeros(b, hidden, dtype=torch.bfloat16, device="cuda")
        xo = torch.empty_like(h)
        flops = 2 * b * k * hidden
        hbm = hidden * k * 2 + b * k * 2
        t_c, t_h = flops / BF16, hbm / HBM
        r = {}
        if symm.multicast:
            tgt = ex.gemm_target(0)
            t_gemm = graph_time_us(lambda: ops.linear_multicast(x, wt, tgt), reps)
            t_bar = graph_time_us(lambda: comm.barrier(symm), reps)
            t_norm = graph_time_us(lambda: comm.add_rmsnorm_slots(ex.local_slots(0), b, h, nw, xo, 1e-5), reps)

            def fused():
                ops.linear_multicast(x, wt, tgt)
                comm.barrier(symm)
                comm.add_rmsnorm_slots(ex.local_slots(0), b, h, nw, xo, 1e-5)

            t_all = graph_time_us(fused, reps)
            nv = (w_ - 1) * b * hidden * 2  # ingress per rank: every other rank's tile
            roof = max(t_c, t_h, nv / NVLINK) * 1e6
            r["slots"] = {"gemm_mcast_us": t_gemm, "barrier_us": t_bar, "add_rmsnorm_us": t_norm, "total_us": t_all,
                          "nvlink_ingress_MB": nv / 1e6, "roofline_us": roof, "fraction": roof / t_all}

            def nvls():
                ops.linear(x, wt, out=ex.slot(1, 0)[:b])
                ex.nvls_reduce(1, b)
                comm.add_rmsnorm_slots(ex.local_slots(1)[1:2], b, h, nw, xo, 1e-5)

            t_nvls = graph_time_us(nvls, reps)
            nv2 = b * hidden * 2  # one reduced copy in, shard multicast
            roof2 = max(t_c, t_h, nv2 / NVLINK) * 1e6
            r["nvls"] = {"total_us": t_nvls, "nvlink_ingress_MB": nv2 / 1e6, "roofline_us": roof2,
                         "fraction": roof2 / t_nvls}

            def gemm_ar():
                ex.gemm_allreduce(x, wt, 0)
                comm.add_rmsnorm_slots(ex.local_slots(0)[1:2], b, h, nw, xo, 1e-5)

            # fb_gemm_bf16_ar_bn*: tiles reduced in the switch and multicast by
            # the GEMM's own epilogue (no barrier or reduce kernel)
            t_ar = graph_time_us(gemm_ar, reps)
            r["gemm_ar"] = {"total_us": t_ar, "nvlink_ingress_MB": nv2 / 1e6, "roofline_us": roof2,
                            "fraction": roof2 / t_ar}
        r["compute_us"], r["hbm_us"] = t_c * 1e6, t_h * 1e6
        out[f"b{b}"] = r
    torch.cuda.synchronize()
    dist.barrier()
    symm.close()
    return out


def ep_path(reps: int) -> dict:
    from ..models.qwen3_moe import Qwen3MoeWeights, qwen3_30b_a3b
    from ..ops import moe as M
    from ..parallel.ep import EPContext
    from .arena import Arena

    cfg = qwen3_30b_a3b()
    cfg.layers = 1
    w_ = dist.get_world_size()
    rows = 512
    ep = EPContext(cfg, rows)
    arena = Arena(None, "8GB")
    wts = Qwen3MoeWeights(cfg, arena, seed=3, ep_rank=ep.rank, ep_size=w_)
    lw = wts.layers[0]

    class St:
        pass

    st = St()
    for name, (shape, dt) in ep.buffers(rows).items():
        setattr(st, name, torch.zeros(shape, dtype=dt, device="cuda"))
    st.ep_ident.copy_(torch.arange(st.ep_ident.numel(), dtype=torch.int32))
    g = torch.Generator(device="cuda").manual_seed(7 + ep.rank)
    logits = torch.randn(rows, cfg.num_experts, device="cuda", generator=g).to(torch.bfloat16)
    st.tids = torch.zeros(rows, cfg.topk, dtype=torch.int32, device="cuda")
    st.tw = torch.zeros(rows, cfg.topk, dtype=torch.float32, device="cuda")
    M.topk(logits, cfg.topk, st.tids, st.tw)
    x = torch.randn(rows, cfg.hidden, device="cuda", generator=g).to(torch.bfloat16)
    h = torch.zeros_like(x)

    class Model:
        @staticmethod
        def _bn_moe(pairs):
            return 64 if pairs > 32 * ep.e_local else 32

    t_all = graph_time_us(lambda: ep.moe(Model, st, x, h, lw, rows), reps)
    k, hd, i = cfg.topk, cfg.hidden, cfg.moe_inter
    pairs = rows * k
    remote = pairs * (w_ - 1) / w_
    nv = remote * (hd + M.kb_pad(hd // 128) * 4 + 4) + remote * hd * 2  # dispatch (fp8 + scales) + combine (bf16)
    flops = 2 * pairs * (hd * 2 * i + i * hd)
    wbytes = ep.e_local * 3 * hd * i  # this rank's fp8 experts
    roof = max(flops / (2 * BF16), wbytes / HBM, nv / NVLINK) * 1e6
    out = {"moe_layer_us": t_all, "nvlink_egress_MB": nv / 1e6, "expert_weight_MB": wbytes / 1e6,
           "roofline_us": roof, "fraction": roof / t_all}
    torch.cuda.synchronize()
    dist.barrier()
    ep.close()
    return out


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reps", type=int, default=20)
    args = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    _peaks()
    res = {"world": dist.get_world_size(), "tp": tp_paths(args.reps), "ep": ep_path(args.reps)}
    if dist.get_rank() == 0:
        print(json.dumps(res))
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
