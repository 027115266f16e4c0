"""Command line for the serving runner: SAVE an archive, LOAD it (with
cold-start timing), or serve a synthetic load.

    python -m foundry_b200.runner.cli save  --archive DIR [--model llama-3-8b] ...
    python -m foundry_b200.runner.cli load  --archive DIR   # prints timings as JSON
    python -m foundry_b200.runner.cli serve --archive DIR --prompts 256 --prompt-len 512 --gen 128

``load`` measures cold start from FOUNDRY_SPAWN_T0_NS (set by the launching
process just before the spawn, as in the reference's vllm/hooks.py:100-112)
to the first generated token of a fresh request.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

T_IMPORT0 = time.time_ns()


def _t0_ns() -> int:
    v = os.environ.get("FOUNDRY_SPAWN_T0_NS")
    return int(v) if v else T_IMPORT0


def build_engine_config(args):
    from ..models import config_by_name
    from .engine import EngineConfig, default_graph_sizes

    try:
        cfg = config_by_name(args.model)
    except KeyError as e:
        raise SystemExit(str(e))
    max_seq = args.prompt_len + args.gen
    pages = -(-max_seq // 64)
    sizes = parse_graph_sizes(args.graph_sizes, args.max_graph_batch)
    return EngineConfig(
        model=cfg, max_batch=max(max(sizes), args.prompts), max_seq_len=max_seq,
        num_blocks=args.prompts * pages + 64, max_prefill_tokens=args.max_prefill_tokens,
        max_prefill_seqs=max(1, args.max_prefill_tokens // args.prompt_len), graph_sizes=sizes,
        region_base=int(args.region_base, 16), region_size=args.region_size, seed=args.seed,
        tp=args.tp, ep=args.ep)


def parse_graph_sizes(spec: str, max_batch: int) -> list[int]:
    """``default``: {1,2,4,8} + 16..max step 16; ``start:stop:step`` (inclusive
    stop), optionally followed by ``+a,b`` extra sizes."""
    from .engine import default_graph_sizes

    if spec == "default":
        return default_graph_sizes(max_batch)
    extra = []
    if "+" in spec:
        spec, more = spec.split("+", 1)
        extra = [int(x) for x in more.split(",") if x]
    a, b, c = (int(x) for x in spec.split(":"))
    return sorted(set(list(range(a, b + 1, c)) + extra))


def init_dist(args) -> None:
    """Process group of a multi-rank (TP / EP) engine: gloo over 127.0.0.1
    bootstraps the symmetric memory; every collective of a step is our own
    kernel."""
    if args.world <= 1:
        return
    import torch.distributed as dist
    from datetime import timedelta

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{args.dist_port}", rank=args.rank,
                            world_size=args.world, timeout=timedelta(seconds=300))


def add_common(p):
    p.add_argument("--archive", required=True)
    p.add_argument("--model", default="llama-3-8b")
    p.add_argument("--prompts", type=int, default=256)
    p.add_argument("--prompt-len", type=int, default=512)
    p.add_argument("--gen", type=int, default=128)
    p.add_argument("--max-graph-batch", type=int, default=1024)
    p.add_argument("--max-prefill-tokens", type=int, default=8192)
    p.add_argument("--region-base", default="0x600000000000")
    p.add_argument("--region-size", default="96GB")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--device", type=int, default=None)
    p.add_argument("--graph-sizes", default="default", help="default | start:stop:step[+a,b]")
    p.add_argument("--tp", type=int, default=1)
    p.add_argument("--ep", type=int, default=1)
    p.add_argument("--rank", type=int, default=0)
    p.add_argument("--world", type=int, default=1)
    p.add_argument("--dist-port", type=int, default=29611)
    p.add_argument("--materialize-all", action="store_true",
                   help="load: after the first token, time until every restored graph has its own executable")


_ENGINES = []


def main(argv=None):
    try:
        return _main(argv)
    finally:
        import torch.distributed as dist

        for eng in _ENGINES:
            eng.close()
        if dist.is_available() and dist.is_initialized():
            dist.destroy_process_group()


def _main(argv=None):
    ap = argparse.ArgumentParser(prog="foundry_b200.runner.cli")
    sub = ap.add_subparsers(dest="cmd", required=True)
    for name in ("save", "load", "serve"):
        add_common(sub.add_parser(name))
    args = ap.parse_args(argv)

    import torch

    marks = {"main_s": time.time_ns()}
    # The (gloo) process group first: it needs no GPU, so it overlaps the CUDA
    # context that FOUNDRY_EARLY_CUDA_INIT may be building on its thread.
    init_dist(args)
    marks["process_group_s"] = time.time_ns()
    if args.device is not None:
        torch.cuda.set_device(args.device)  # creates (or waits for) the device's primary context
    marks["cuda_context_s"] = time.time_ns()
    from . import persist

    marks["runner_import_s"] = time.time_ns()

    if args.cmd == "save":
        from .engine import LLMEngine

        t0 = time.perf_counter()
        eng = LLMEngine(build_engine_config(args))
        _ENGINES.append(eng)
        st = persist.save(eng, args.archive)
        st["engine_setup_s"] = eng.setup_s
        st["wall_s"] = time.perf_counter() - t0
        print(json.dumps({"save": {k: v for k, v in st.items() if k != "engine"}}))
        return 0

    if args.cmd == "load":
        eng, timings = persist.load(args.archive)
        _ENGINES.append(eng)
        marks["archive_load_s"] = time.time_ns()
        # First token of a fresh request through the restored engine.
        g = torch.Generator().manual_seed(args.seed + 7)
        prompt = torch.randint(0, eng.ecfg.model.vocab, (args.prompt_len,), generator=g).tolist()
        reqs = eng.add_requests([prompt], max_new_tokens=2)
        eng.prefill(reqs)
        first = time.time_ns()
        b = eng.start_decode(reqs)
        eng.decode_step(b)
        second = time.time_ns()
        eng.release(reqs)
        if args.materialize_all:
            # the first decode step started materialising every restored graph
            # on a background thread (largest batch first); wait for the end
            eng.wait_materialized()
            eng.materialize_graphs(background=False)  # no-op for graphs already done
            timings["materialize_all_s_after_first_token"] = (time.time_ns() - first) / 1e9
        timings.update({
            "cold_start_first_token_s": (first - _t0_ns()) / 1e9,
            "cold_start_first_decode_token_s": (second - _t0_ns()) / 1e9,
            "python_import_s": (T_IMPORT0 - _t0_ns()) / 1e9 if os.environ.get("FOUNDRY_SPAWN_T0_NS") else None,
        })
        # Where the time to the first token went, step by step from the
        # end of the imports (seconds per step, in order).
        marks["first_token_s"] = first
        prev, steps = T_IMPORT0, {}
        for k, t in marks.items():
            steps[k] = round((t - prev) / 1e9, 4)
            prev = t
        timings["cold_start_steps_s"] = steps
        from .. import _early_cuda

        timings["early_cuda_context"] = _early_cuda.result()
        print(json.dumps({"load": timings}))
        return 0

    if args.cmd == "serve":
        eng, timings = persist.load(args.archive)
        _ENGINES.append(eng)
        g = torch.Generator().manual_seed(args.seed + 11)
        prompts = torch.randint(0, eng.ecfg.model.vocab, (args.prompts, args.prompt_len), generator=g).tolist()
        t0 = time.perf_counter()
        outs = eng.generate(prompts, args.gen)
        dt = time.perf_counter() - t0
        print(json.dumps({"serve": {"requests": len(outs), "gen_tokens": sum(map(len, outs)), "wall_s": dt,
                                    "restore": timings}}))
        return 0
    return 1


if __name__ == "__main__":
    sys.exit(main())
