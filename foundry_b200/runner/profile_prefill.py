"""Prefill timing at serving shape (profiling driver): ``--prompts`` random
prompts of ``--prompt-len`` tokens through the engine's packed, chunked
prefill; prints the device time per run and tokens/s. Under ncu, capture the
attention kernel with ``-k regex:fb_prefill_attn_tc``.

    python -m foundry_b200.runner.profile_prefill --model llama-3-8b@2l --prompts 16 --prompt-len 2048
"""

from __future__ import annotations

import argparse
import json

import torch


def attn_only(args) -> int:
    """Device time of ops.prefill_attention over packed prompts (CUDA events,
    after one warm-up call), causal FLOPs and the fraction of the measured
    bf16 tensor peak."""
    import math
    import os

    from .. import ops
    from ..models import config_by_name
    from ..ops.attention import PREFILL_TILE, prefill_tiles

    cfg = config_by_name(args.model)
    hq, hkv, d = cfg.n_q, cfg.n_kv, cfg.head_dim
    n, L = args.prompts, args.prompt_len
    t = n * L
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(t, hq * d, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(t, hkv * d, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(t, hkv * d, device="cuda", generator=g).to(torch.bfloat16)
    out = torch.empty(t, hq * d, device="cuda", dtype=torch.bfloat16)
    cu = torch.tensor([i * L for i in range(n + 1)], dtype=torch.int32, device="cuda")
    ts, tst = prefill_tiles([L] * n, PREFILL_TILE[args.impl])
    ts = torch.tensor(ts, dtype=torch.int32, device="cuda")
    tst = torch.tensor(tst, dtype=torch.int32, device="cuda")
    run = lambda: ops.prefill_attention(q, k, v, out, cu, ts, tst, hq, hkv, impl=args.impl)  # noqa: E731
    run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.runs):
        run()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000 / args.runs
    flops = 4 * d * hq * n * (L * (L + 1) / 2)  # QK^T and PV over the causal triangle
    peak = 1654e12
    try:
        with open(os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")) as f:
            peak = float(json.load(f)["bf16_tflops"]) * 1e12
    except (OSError, KeyError, ValueError):
        pass
    print(json.dumps({"impl": args.impl, "prompts": n, "prompt_len": L, "heads": [hq, hkv], "us": round(us, 1),
                      "tflops": round(flops / us / 1e6, 1), "frac_of_measured_bf16": round(flops / us / 1e6 / (peak / 1e12), 3),
                      "status": ops.status("prefill_tc")}))
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama-3-8b@2l")
    ap.add_argument("--prompts", type=int, default=16)
    ap.add_argument("--prompt-len", type=int, default=2048)
    ap.add_argument("--runs", type=int, default=2)
    ap.add_argument("--attn-only", action="store_true",
                    help="time the causal prefill attention kernel alone on random packed q/k/v "
                         "(--prompts x --prompt-len tokens, the model's head counts)")
    ap.add_argument("--impl", default="tc", help="prefill attention implementation for --attn-only")
    args = ap.parse_args()
    if args.attn_only:
        return attn_only(args)

    from ..models import config_by_name
    from .engine import EngineConfig, LLMEngine

    cfg = config_by_name(args.model)
    ecfg = EngineConfig(model=cfg, max_batch=max(16, args.prompts), max_seq_len=args.prompt_len + 8,
                        max_prefill_tokens=8192, max_prefill_seqs=max(1, 8192 // args.prompt_len), graph_sizes=[16],
                        region_base=None, region_size="64GB")
    eng = LLMEngine(ecfg)
    g = torch.Generator().manual_seed(3)
    times = []
    for _ in range(args.runs):
        prompts = torch.randint(0, cfg.vocab, (args.prompts, args.prompt_len), generator=g).tolist()
        reqs = eng.add_requests(prompts, max_new_tokens=1)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        eng.prefill(reqs)
        e1.record()
        torch.cuda.synchronize()
        eng.release(reqs)
        times.append(e0.elapsed_time(e1))
    tokens = args.prompts * args.prompt_len
    print(json.dumps({"model": args.model, "tokens": tokens, "ms": times, "tok_per_s": tokens / (min(times) / 1e3)}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
