"""Decode-attention timing at serving shape, one kernel at a time.

    python -m foundry_b200.runner.profile_attention --batch 256 --ctx 530 --impl tc
    python -m foundry_b200.runner.profile_attention --batch 512 --ctx 1100 --heads 32,4 --impl tc,tc3,simt

Builds a paged KV cache (pages in random order, so page reads are scattered
the way a serving cache's are), one query per sequence and per-sequence
lengths of ``--ctx`` tokens (or uniform in ``[ctx - jitter, ctx]``), then
times ``--iters`` calls of ``ops.decode_attention`` per implementation with
CUDA events on the launching stream after ``--warmup`` calls. The cache is
larger than L2 at serving shapes, so every call reads it from HBM.

Prints one JSON line per implementation: microseconds per call, algorithmic
bytes (K and V of every live token, plus Q and the output), achieved GB/s
and the fraction of the measured HBM copy bandwidth, and the largest
difference from the first implementation's output (``--check`` also compares
with an fp32 PyTorch reference on the first 8 sequences).
"""

from __future__ import annotations

import argparse
import json
import math
import os

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def measured_hbm_gbs() -> float:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 6650.0


def reference(q, kc, vc, tables, lens, scale):
    """fp32 paged attention for each sequence (GQA)."""
    b, hq, d = q.shape
    hkv, page = kc.shape[1], kc.shape[2]
    g = hq // hkv
    out = torch.empty(b, hq, d, dtype=torch.float32, device=q.device)
    for i in range(b):
        n = int(lens[i])
        pages = tables[i, : math.ceil(n / page)].long()
        k = kc[pages].permute(1, 0, 2, 3).reshape(hkv, -1, d)[:, :n].float()
        v = vc[pages].permute(1, 0, 2, 3).reshape(hkv, -1, d)[:, :n].float()
        qq = q[i].float().view(hkv, g, d)
        p = torch.softmax(qq @ k.transpose(1, 2) * scale, dim=-1)
        out[i] = (p @ v).reshape(hq, d)
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--ctx", type=int, default=530)
    ap.add_argument("--jitter", type=int, default=0, help="lengths uniform in [ctx - jitter, ctx]")
    ap.add_argument("--heads", default="32,8", help="query heads,kv heads")
    ap.add_argument("--impl", default="tc", help="comma list of tc, tc3, simt")
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--check", action="store_true")
    ap.add_argument("--splits", type=int, default=0,
                    help="force this many KV splits per sequence (0 = the planner's choice)")
    a = ap.parse_args(argv)
    from foundry_b200 import ops
    from foundry_b200.ops.attention import DecodeWorkspace, decode_splits

    hq, hkv = (int(x) for x in a.heads.split(","))
    b, d, page = a.batch, 128, 64
    max_pages = math.ceil(a.ctx / page)
    max_pages += max_pages % 2
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(0)
    blocks = b * max_pages
    kc = torch.randn(blocks, hkv, page, d, device=dev, generator=gen, dtype=torch.bfloat16)
    vc = torch.randn(blocks, hkv, page, d, device=dev, generator=gen, dtype=torch.bfloat16)
    tables = torch.randperm(blocks, device=dev, generator=gen).to(torch.int32).view(b, max_pages)
    lo = max(1, a.ctx - a.jitter)
    lens = torch.randint(lo, a.ctx + 1, (b,), device=dev, generator=gen, dtype=torch.int32)
    q = torch.randn(b, hq, d, device=dev, generator=gen, dtype=torch.bfloat16)
    scale = 1.0 / math.sqrt(d)
    splits = decode_splits(b, hkv, max_pages)
    if a.splits:
        cps = math.ceil(math.ceil(max_pages / 2) / a.splits)
        splits = (math.ceil(math.ceil(max_pages / 2) / cps), 2 * cps)
    ws = DecodeWorkspace(b, hq, max(splits[0], 1), device=dev)
    live = int(lens.sum())
    algo_bytes = live * hkv * d * 2 * 2 + 2 * q.numel() * 2
    peak = measured_hbm_gbs()
    first = None
    for impl in a.impl.split(","):
        out = torch.empty_like(q)
        for _ in range(a.warmup):
            ops.decode_attention(q, kc, vc, tables, lens, out, max_pages, ws, scale=scale, splits=splits, impl=impl)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.iters):
            ops.decode_attention(q, kc, vc, tables, lens, out, max_pages, ws, scale=scale, splits=splits, impl=impl)
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1000 / a.iters
        row = {"impl": impl, "batch": b, "ctx": a.ctx, "jitter": a.jitter, "heads": [hq, hkv], "splits": splits[0],
               "us": round(us, 2), "algo_MB": round(algo_bytes / 1e6, 1),
               "GBps": round(algo_bytes / us / 1e3, 1), "frac_of_measured_hbm": round(algo_bytes / us / 1e3 / peak, 3)}
        if first is None:
            first = out.float()
        else:
            row["max_diff_vs_first"] = float((out.float() - first).abs().max())
        if a.check:
            n = min(8, b)
            ref = reference(q[:n], kc, vc, tables[:n], lens[:n], scale)
            row["max_err_vs_fp32"] = float((out[:n].float() - ref).abs().max())
        print(json.dumps(row), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
