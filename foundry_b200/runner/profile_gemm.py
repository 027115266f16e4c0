"""Times the bf16 decode GEMM variants on the shapes of a model's decode step.

    python -m foundry_b200.runner.profile_gemm --model llama-3-8b --tokens 256
    python -m foundry_b200.runner.profile_gemm --model llama-3-8b --tokens 256 --variants plan,pair --check

For every linear layer of one decoder layer (+ lm_head) at ``--tokens``
tokens it prints one JSON line per variant:
- ``plan``: the planner's choice (one-SM tiles, split-K, stream-K);
- ``pair``: two-SM ``cta_group::2`` tiles with the same tile width;
- ``pf<N>``: the planner's plan with an L2 prefetch lead of N k-blocks;
- ``bn<B>s<S>[m<T>]``: one-SM tiles of B tokens, S splits, T weight tiles per
  unit (default 1);
- ``pair<B>s<S>``: two-SM tiles of B tokens with S splits;
- ``sk<B>``: stream-K over one-SM tiles of B tokens;
- ``cublas``: ``torch.matmul`` on the same operands (cuBLAS), for comparison;
- ``swiglu`` (gate_up only): the fused gate/up GEMM whose epilogue writes
  silu(gate) * up (``fb_gemm_bf16_bn*_m2``, one 128-feature unit per CTA);
- ``swiglusk`` (gate_up only): its stream-K form (``fb_gemm_swiglu_sk_bn256``,
  every CTA an equal share of the unit x k-block iterations; off in the
  decode step unless FOUNDRY_SWIGLU_SK=1).
``--ops`` restricts the run to some layers (e.g. ``gate_up,lm_head``).

Each line gives the plan (tile width, splits, grid) and the mean time of
``--iters`` back-to-back launches (CUDA events, after ``--warmup``);
``--pdl`` launches them with programmatic dependent launch as in the decode
step, ``--flush`` (with ``--graph``) evicts L2 before each launch.
Weights larger than the 126 MB L2 (Llama-3-8B gate_up, down, lm_head) stream
from HBM on every launch. Smaller ones (qkv 50 MB, o 34 MB) may partly stay
in L2 across back-to-back launches, which they do not inside a decode step.
With ``--check`` each variant's output is compared against fp32.
"""

from __future__ import annotations

import argparse
import contextlib
import dataclasses
import json
import sys


def shapes(cfg, tokens: int):
    h, d = cfg.hidden, cfg.head_dim
    out = [("qkv", tokens, cfg.qkv_dim, h), ("o", tokens, h, cfg.n_q * d)]
    if getattr(cfg, "inter", 0):
        out += [("gate_up", tokens, 2 * cfg.inter, h), ("down", tokens, h, cfg.inter)]
    out.append(("lm_head", tokens, cfg.vocab, h))
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="foundry_b200.runner.profile_gemm")
    ap.add_argument("--model", default="llama-3-8b")
    ap.add_argument("--tokens", type=int, default=256)
    ap.add_argument("--variants", default="plan,pair")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--check", action="store_true")
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--ops", default="", help="comma-separated subset of qkv,o,gate_up,down,lm_head")
    ap.add_argument("--graph", action="store_true",
                    help="time one CUDA-graph replay of --iters launches (no host launch overhead)")
    ap.add_argument("--shape", default="", help="n,k: one custom weight shape instead of the model's layers")
    ap.add_argument("--pdl", action="store_true",
                    help="launch with programmatic dependent launch, as inside the decode step")
    ap.add_argument("--flush", action="store_true",
                    help="with --graph: write a 256 MB buffer before every launch (weights cold in L2, as in "
                         "the decode step) and report the time minus that of the flushes alone")
    a = ap.parse_args(argv)

    import torch

    from .. import ops
    from ..models import config_by_name
    from ..ops import gemm as G

    torch.cuda.set_device(a.device)
    cfg = config_by_name(a.model)
    sms = G._rt.sm_count()
    gen = torch.Generator(device="cuda").manual_seed(0)
    only = set(filter(None, a.ops.split(",")))
    todo = shapes(cfg, a.tokens)
    if a.shape:
        n_, k_ = (int(v) for v in a.shape.split(","))
        todo = [("custom", a.tokens, n_, k_)]
    flush_buf = torch.empty(64 << 20, dtype=torch.float32, device="cuda") if a.flush else None
    for name, t, n, k in todo:
        if only and name not in only:
            continue
        x = (torch.randn(t, k, device="cuda", generator=gen) * 0.5).to(torch.bfloat16)
        w = (torch.randn(n, k, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
        pb = G.PartialBuffer(G.MAX_SPLITS * t * n)
        out = torch.empty(t, n, dtype=torch.bfloat16, device="cuda")
        ref = (x.float() @ w.float().T) if a.check else None
        base = G.plan(t, n, k)
        for v in a.variants.split(","):
            cublas = v == "cublas"  # torch.matmul (cuBLAS / cuBLASLt) on the same operands, for comparison
            swiglu = v in ("swiglu", "swiglusk")
            swiglu_sk = None
            if v in ("plan", "cublas"):
                p = base
            elif swiglu:
                if name != "gate_up":
                    continue
                p = G.plan_swiglu(t, n // 2, k) if v == "swiglu" else G.plan_swiglu_sk(t, n // 2, k, force=True)
                if p is None:
                    continue
                act = torch.empty(t, n // 2, dtype=torch.bfloat16, device="cuda")
                if p.streamk:
                    ws_n, fl_n = G.swiglu_sk_sizes(n // 2)
                    swiglu_sk = G.StreamKBuffer(torch.empty(ws_n, dtype=torch.float32, device="cuda"),
                                                torch.zeros(fl_n, dtype=torch.int32, device="cuda"))
            elif v == "pair":
                if not base.swap or n < 256:
                    continue
                p = G.pair_plan(n, t, k, max(64, base.bn), sms, pf=base.pf)
            elif v.startswith("pf"):
                p = dataclasses.replace(base, pf=int(v[2:]))
            elif v.startswith("bn"):
                bn, rest = v[2:].split("s")
                sp, mt = (rest.split("m") + ["1"])[:2]
                bn, sp, mt = int(bn), int(sp), int(mt)
                units = -(-n // (128 * mt)) * -(-t // bn) * sp if base.swap else 0
                p = dataclasses.replace(base, bn=bn, splits=sp, mt=mt, grid=min(units, sms), streamk=False,
                                        pair=False)
            elif v.startswith("pair") and v != "pair":
                bn, sp = (int(x) for x in v[4:].split("s"))
                tiles = -(-n // 256) * -(-t // bn)
                p = G.Plan(bn=bn, splits=sp, grid=2 * min(tiles * sp, sms // 2), swap=True, pf=base.pf,
                           pair=True)
            elif v.startswith("sk"):
                bn = int(v[2:])
                p = dataclasses.replace(base, bn=bn, splits=1, mt=1, grid=sms, streamk=True, pair=False)
            else:
                raise SystemExit(f"unknown variant {v!r}")

            skb = None
            if p.streamk and not swiglu:
                skb = G.StreamKBuffer(torch.empty(sms * 128 * 256, dtype=torch.float32, device="cuda"),
                                      torch.zeros(sms * 8, dtype=torch.int32, device="cuda"))

            def run():
                if cublas:
                    return torch.matmul(x, w.T, out=out)
                with G._rt.pdl() if a.pdl else contextlib.nullcontext():
                    if swiglu:
                        return G.linear_swiglu(x, w, act, plan_override=p, sk=swiglu_sk)
                    return G.linear(x, w, out=out, partials=pb if p.splits > 1 else None, plan_override=p,
                                    streamk=skb)

            for _ in range(a.warmup):
                run()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            flush_us = 0.0
            if a.graph:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    for _ in range(a.iters):
                        if a.flush:
                            flush_buf.fill_(1.0)
                        r = run()
                g.replay()
                torch.cuda.synchronize()
                e0.record()
                g.replay()
                e1.record()
                if a.flush:
                    gf = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(gf):
                        for _ in range(a.iters):
                            flush_buf.fill_(1.0)
                    gf.replay()
                    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    torch.cuda.synchronize()
                    f0.record()
                    gf.replay()
                    f1.record()
                    torch.cuda.synchronize()
                    flush_us = f0.elapsed_time(f1) * 1000 / a.iters
            else:
                e0.record()
                for _ in range(a.iters):
                    r = run()
                e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1000 / a.iters - flush_us
            line = {"op": name, "tokens": t, "n": n, "k": k, "variant": v,
                    "kernel": "cublas" if cublas else (f"fb_gemm_swiglu_sk_bn{p.bn}" if swiglu_sk else p.kernel),
                    "bn": p.bn,
                    "splits": p.splits, "grid": p.grid, "us": round(us, 1),
                    "weight_tbps": round(n * k * 2 / (us * 1e-6) / 1e12, 2),
                    "tflops": round(2 * t * n * k / (us * 1e-6) / 1e12, 1)}
            if a.check:
                y = (r.buf[: r.splits * r.stride].view(r.splits, t, n).sum(0) if isinstance(r, G.Partial)
                     else r.float())
                want = ref
                if swiglu:  # [gate; up] rows: silu(x @ gate.T) * (x @ up.T)
                    want = torch.nn.functional.silu(ref[:, : n // 2]) * ref[:, n // 2:]
                line["max_err"] = round((y - want).abs().max().item(), 4)
            line["status"] = ops.status("gemm_bf16")
            print(json.dumps(line), flush=True)
            if line["status"]:
                return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
