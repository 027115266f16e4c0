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


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama-3-8b@2l")
    ap.add_argument("--prompts", type=int, default=16)
    ap.add_argument("--prompt-len", type=int, default=2048)
    ap.add_argument("--runs", type=int, default=2)
    args = ap.parse_args()

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
