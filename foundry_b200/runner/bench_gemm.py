"""GEMM microbenchmark: times ``ops.linear`` for decode/prefill shapes and
tile configurations with CUDA events (median of repeated launches; weights
rotate through enough copies to exceed L2 so every launch streams from HBM).

    python -m foundry_b200.runner.bench_gemm --shapes 256x28672x4096 --sweep
"""

from __future__ import annotations

import argparse
import itertools
import json
import math

import torch


def time_linear(x, ws, plan, pb, reps=20):
    from foundry_b200 import ops

    out = torch.empty(x.shape[0], ws[0].shape[0], dtype=torch.bfloat16, device="cuda")
    for w in ws[:2]:
        ops.linear(x, w, out=out, partials=pb, plan_override=plan)
    torch.cuda.synchronize()
    times = []
    for i in range(reps):
        w = ws[i % len(ws)]
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        ops.linear(x, w, out=out, partials=pb, plan_override=plan)
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1) * 1e3)
    times.sort()
    return times[len(times) // 2]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default="256x6144x4096,256x4096x4096,256x28672x4096,256x4096x14336,256x128256x4096")
    ap.add_argument("--sweep", action="store_true")
    ap.add_argument("--pf", default="0,8,16,32")
    args = ap.parse_args()
    from foundry_b200 import ops
    from foundry_b200.ops.gemm import Plan, plan

    res = []
    for shp in args.shapes.split(","):
        t, n, k = map(int, shp.split("x"))
        nbytes = n * k * 2
        copies = max(2, math.ceil(300e6 / nbytes))
        ws = [torch.randn(n, k, device="cuda").to(torch.bfloat16) * 0.02 for _ in range(copies)]
        x = torch.randn(t, k, device="cuda").to(torch.bfloat16)
        pb = ops.PartialBuffer(8 * t * n)
        auto = plan(t, n, k)
        cands = [auto]
        if args.sweep:
            cands = []
            for bn, mt, s, pf in itertools.product((64, 128, 256), (1, 2), (1, 2, 3, 4, 8), map(int, args.pf.split(","))):
                if auto.swap and bn < 64 and t > 64:
                    continue
                if not auto.swap and bn < 128:
                    continue
                units = math.ceil((n if auto.swap else t) / (128 * mt)) * math.ceil((t if auto.swap else n) / bn) * s
                cands.append(Plan(bn=bn, splits=s, grid=min(units, 148), swap=auto.swap, mt=mt, pf=pf))
        for p in cands:
            us = time_linear(x, ws, p, pb)
            gbs = (nbytes + t * k * 2) / (us * 1e-6) / 1e9
            res.append({"shape": shp, "bn": p.bn, "mt": p.mt, "splits": p.splits, "pf": p.pf, "us": round(us, 2),
                        "GBps": round(gbs), "auto": p is auto})
            print(json.dumps(res[-1]), flush=True)
        best = min((r for r in res if r["shape"] == shp), key=lambda r: r["us"])
        print("BEST", json.dumps(best), flush=True)
        del ws


if __name__ == "__main__":
    main()
