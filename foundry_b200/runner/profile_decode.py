"""Per-kernel timing of one decode step at serving shape (profiling driver).

Builds the engine without persistence, fills the KV cache with random data
and sets every sequence to ``--ctx`` cached tokens (no prefill), then runs
``--warmup`` eager decode steps followed by ``--steps`` profiled ones. Run it
plain to get per-op CUDA-event timings, or under ncu to capture kernels:

    python -m foundry_b200.runner.profile_decode --batch 256 --ctx 576
    ncu --metrics gpu__time_duration.sum --clock-control none -k regex:fb_ \
        -s <warmup launches> -c <launches> --csv python -m foundry_b200.runner.profile_decode ...
"""

from __future__ import annotations

import argparse
import json
import time

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama-3-8b")
    ap.add_argument("--layers", type=int, default=None, help="override layer count (smaller captures)")
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--ctx", type=int, default=576)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1)
    ap.add_argument("--ops", action="store_true", help="time each op with CUDA events (eager)")
    ap.add_argument("--attn", default=None, help="decode attention implementation (tc1, tc3, simt)")
    args = ap.parse_args()
    if args.attn:
        from foundry_b200 import ops as _ops

        _orig = _ops.decode_attention
        _ops.decode_attention = lambda *a, **k: _orig(*a, impl=args.attn, **k)

    from ..models import config_by_name
    from .engine import PAGE, EngineConfig, LLMEngine

    cfg = config_by_name(args.model)
    if args.layers:
        cfg.layers = args.layers
    max_seq = args.ctx + args.warmup + args.steps + 8
    pages = -(-max_seq // PAGE)
    ecfg = EngineConfig(model=cfg, max_batch=args.batch, max_seq_len=max_seq, num_blocks=args.batch * pages,
                        max_prefill_tokens=256, max_prefill_seqs=1, graph_sizes=[args.batch], region_base=None)
    eng = LLMEngine(ecfg)
    from .. import ops

    for kc, vc in zip(eng.k_cache, eng.v_cache):
        ops.init_normal_(kc.view(-1), seed=7, std=1.0)
        ops.init_normal_(vc.view(-1), seed=8, std=1.0)
    b = args.batch
    st = eng.state
    tables = torch.arange(b * pages, dtype=torch.int32).view(b, pages)
    st.block_tables[:b, :pages].copy_(tables)
    st.seq_lens[:b].fill_(args.ctx)
    st.active[:b].fill_(1)
    st.input_ids[:b].copy_(torch.randint(0, cfg.vocab, (b,), dtype=torch.int32))
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        eng.model.decode(st, b)
    torch.cuda.synchronize()
    if args.ops:
        times = {}
        orig = {}
        for name in ("rmsnorm", "linear", "rope_kv_write", "decode_attention", "silu_mul", "embedding", "argmax",
                     "decode_advance"):
            fn = getattr(ops, name)
            orig[name] = fn

            def wrap(*a, _n=name, _f=fn, **k):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                r = _f(*a, **k)
                e1.record()
                torch.cuda.synchronize()
                key = _n
                if _n == "linear":
                    key = f"linear[{a[1].shape[0]}x{a[1].shape[1]}]"
                times.setdefault(key, []).append(e0.elapsed_time(e1))
                return r

            setattr(ops, name, wrap)
        import foundry_b200.models.llama as lm

        lm.ops = ops
        eng.model.decode(st, b)
        for name, fn in orig.items():
            setattr(ops, name, fn)
        out = {k: {"n": len(v), "ms_each": sum(v) / len(v), "ms_total": sum(v)} for k, v in times.items()}
        print(json.dumps({"per_op": out, "step_ms_sum": sum(x["ms_total"] for x in out.values())}, indent=1))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        eng.model.decode(st, b)
    e1.record()
    torch.cuda.synchronize()
    print(json.dumps({"eager_step_ms": e0.elapsed_time(e1) / args.steps, "batch": b, "ctx": args.ctx}))


if __name__ == "__main__":
    main()
