"""Headline benchmark: restored-graph decode throughput of the Llama-3-8B-shaped
serving load (256 prompts x 512 random tokens, greedy) on N GPUs (DP: one
full engine per GPU, weak scaling), plus the persistence numbers of the same
run: graph capture + SAVE, fresh-process cold start to first token, and
restore time of the 67 decode graphs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl foundry|reference|torch]

For N > 1 launch with torch.distributed.run (one rank per GPU). Rank 0 prints
one JSON line. ``value`` is the device-timed decode rate (CUDA events around
K back-to-back restored-graph steps, max over ranks, summed over ranks as
tokens / slowest rank's time); ``e2e`` is the same metric through the public
engine API with a pinned-host H2D of each step's input tokens and a D2H of
the sampled tokens every step. ``--impl torch`` runs the same decode step in
stock PyTorch (cuBLAS GEMMs, SDPA attention) under torch.cuda.graph, as a
same-box comparison.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

REF_UNAVAILABLE = (
    "reference build needs Boost>=1.83 (CMakeLists.txt:9 find_package(Boost)); Boost is not on this image and "
    "there is no network; pip install of the reference fails at its CMake configure step"
)


# Serving loads of the benchmark configurations: prompts (per GPU for dp/ep,
# per job for tp), prompt and output lengths, persisted decode graph sizes,
# region size and parallel mode.
PRESETS = {
    "llama-3-8b": dict(batch=256, prompt_len=512, gen=128, graph_sizes="default", region="96GB", parallel="dp"),
    "qwen3-30b-a3b": dict(batch=512, prompt_len=1024, gen=256, graph_sizes="2:512:2", region="170GB",
                          parallel="ep"),
    "llama-3-70b": dict(batch=1024, prompt_len=2048, gen=256, graph_sizes="default", region="170GB",
                        parallel="tp"),
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="foundry", choices=["foundry", "reference", "torch", "vllm"],
                    help="torch: the same decode step in stock PyTorch (cuBLAS, SDPA) under torch.cuda.graph; "
                         "vllm: upstream vLLM on the same shape (dummy weights, no tokenizer)")
    ap.add_argument("--model", default="llama-3-8b")
    ap.add_argument("--batch", type=int, default=None, help="prompts per GPU (dp/ep) or per job (tp)")
    ap.add_argument("--prompt-len", type=int, default=None)
    ap.add_argument("--gen", type=int, default=None)
    ap.add_argument("--graph-sizes", default=None)
    ap.add_argument("--region-size", default=None)
    ap.add_argument("--parallel", default=None, choices=["dp", "tp", "ep"])
    ap.add_argument("--workdir", default=None)
    ap.add_argument("--skip-cold-start", action="store_true")
    args = ap.parse_args()
    base = args.model.split("@")[0]
    preset = PRESETS.get(base, PRESETS["llama-3-8b"])
    for k, v in (("batch", "batch"), ("prompt_len", "prompt_len"), ("gen", "gen"), ("graph_sizes", "graph_sizes"),
                 ("region_size", "region"), ("parallel", "parallel")):
        if getattr(args, k) is None:
            setattr(args, k, preset[v])
    return args


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.device)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def run_cli(cmd: list[str], env_extra: dict | None = None, timeout: int = 1800) -> dict:
    # The runner gets its rank and rendezvous from its own arguments; the
    # launcher's variables (TORCHELASTIC_USE_AGENT_STORE in particular, which
    # makes rank 0 join the agent's store instead of hosting one) must not leak.
    env = {k: v for k, v in os.environ.items()
           if not k.startswith(("TORCHELASTIC_", "TORCH_ELASTIC")) and k not in (
               "RANK", "LOCAL_RANK", "WORLD_SIZE", "LOCAL_WORLD_SIZE", "GROUP_RANK", "ROLE_RANK", "ROLE_WORLD_SIZE",
               "MASTER_ADDR", "MASTER_PORT", "GROUP_WORLD_SIZE", "ROLE_NAME")}
    env.update(env_extra or {})
    env["PYTHONPATH"] = ROOT + os.pathsep + env.get("PYTHONPATH", "")
    res = subprocess.run([sys.executable, "-m", "foundry_b200.runner.cli", *cmd], env=env, capture_output=True,
                         text=True, timeout=timeout)
    if res.returncode != 0:
        raise RuntimeError(f"runner {cmd[0]} failed:\n{res.stdout[-4000:]}\n{res.stderr[-4000:]}")
    for line in reversed(res.stdout.strip().splitlines()):
        if line.startswith("{"):
            return json.loads(line)
    raise RuntimeError(f"runner {cmd[0]} printed no JSON:\n{res.stdout[-2000:]}")


def run_torch_baseline(args, rank: int, world: int, local: int) -> int:
    """Same model, batch and graph sizes as the foundry arm, in stock PyTorch
    (foundry_b200/runner/torch_baseline.py); data-parallel over the ranks."""
    import torch
    import torch.distributed as dist

    from foundry_b200.runner.cli import parse_graph_sizes
    from foundry_b200.runner.torch_baseline import run

    gen = max(args.gen, 1 + args.warmup + 2 * args.steps + 2)
    sizes = parse_graph_sizes(args.graph_sizes, 1024)
    sampler = ClockSampler(local)
    sampler.start()
    r = run(args.model, args.batch, args.prompt_len, gen, args.steps, args.warmup, sizes, device=local)
    clocks = sampler.stop()
    t = torch.tensor([r["dev_ms"], r["capture_s"]], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dev_ms, capture_s = t.tolist()
    tokens = args.batch * world * args.steps
    if rank == 0:
        print(json.dumps({
            "impl": "torch",
            "metric": f"graph decode tok/s ({args.model} shape, {r['num_graphs']} torch.cuda.graph decode graphs)",
            "value": round(tokens / (dev_ms / 1e3), 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random token ids, random-init N(0,0.02) weights, KV cache filled with random "
                    "values of the prompt length instead of a prefill)",
            "config": {"model": args.model, "global_batch": args.batch * world, "seq_len": args.prompt_len + gen,
                       "prompt_len": args.prompt_len, "parallelism": f"dp{world}", "graphs_per_rank": r["num_graphs"],
                       "kernels": r["kernels_note"],
                       "l2": "inputs larger than L2 (all weights + the KV cache are read every step)"},
            "clocks": clocks,
            "capture_s": round(capture_s, 2),
        }))
    if world > 1:
        dist.destroy_process_group()
    return 0


def run_vllm_baseline(args, rank: int, world: int, local: int) -> int:
    """Upstream vLLM on the same model shape, batch and graph sizes, one engine
    per GPU (data parallel over the ranks; foundry_b200/runner/vllm_baseline.py)."""
    import torch
    import torch.distributed as dist

    from foundry_b200.runner.cli import parse_graph_sizes
    from foundry_b200.runner.vllm_baseline import run

    workdir = args.workdir or f"/tmp/foundry_vllm_{os.environ.get('MASTER_PORT', os.getpid())}_{rank}"
    # vLLM's engine process is spawned with this environment: show it this rank's GPU only
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    ids = [x for x in visible.split(",") if x] if visible else [str(i) for i in range(torch.cuda.device_count())]
    os.environ["CUDA_VISIBLE_DEVICES"] = ids[local]
    sampler = ClockSampler(local)
    sampler.start()
    r = run(args.model, args.batch, args.prompt_len, args.gen, parse_graph_sizes(args.graph_sizes, 1024), workdir)
    clocks = sampler.stop()
    t = torch.tensor([r["decode_s"]], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    decode_s = float(t.item())
    if rank == 0:
        tokens = r["decode_tokens"] * world
        print(json.dumps({
            "impl": "vllm", "metric": f"decode tok/s ({args.model} shape, upstream vLLM, FULL_DECODE_ONLY graphs)",
            "value": round(tokens / decode_s, 1), "unit": "tokens/s", "n_gpus": world,
            "ms_per_step": round(r["ms_per_step"], 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp8-block + bf16" if "qwen3" in args.model else "bf16",
            "data": "synthetic (random token-id prompts, dummy weights)",
            "timing": "host wall clock around blocking generate() calls with device syncs: decode = generate(gen) "
                      "- generate(1)",
            "config": {"model": args.model, "global_batch": args.batch * world, "prompt_len": args.prompt_len,
                       "gen_len": args.gen, "parallelism": f"dp{world}"},
            "startup_s": round(r["startup_s"], 2), "prefill_s": round(r["prefill_s"], 3), "clocks": clocks,
        }))
    if world > 1:
        dist.destroy_process_group()
    return 0


def main():
    args = parse()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": REF_UNAVAILABLE}))
        return 0

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    if args.impl == "torch":
        return run_torch_baseline(args, rank, world, local)
    if args.impl == "vllm":
        return run_vllm_baseline(args, rank, world, local)

    gen = max(args.gen, 1 + args.warmup + 2 * args.steps + 2)
    mode = args.parallel if world > 1 else "dp"
    port = int(os.environ.get("MASTER_PORT", 29500))
    workdir = args.workdir or f"/tmp/foundry_bench_{os.environ.get('MASTER_PORT', os.getpid())}"
    # dp: independent engines, one archive per rank; tp / ep: one multi-rank
    # engine whose archive holds a rank_<r> folder per rank
    archive = os.path.join(workdir, f"rank_{rank}") if mode == "dp" else workdir
    common = ["--archive", archive, "--model", args.model, "--prompts", str(args.batch), "--prompt-len",
              str(args.prompt_len), "--gen", str(gen), "--device", str(local), "--graph-sizes", args.graph_sizes,
              "--region-size", args.region_size]
    if mode in ("tp", "ep"):
        common += [f"--{mode}", str(world), "--rank", str(rank), "--world", str(world)]

    # 1) SAVE in a fresh process: capture the decode graphs and write the archive.
    t0 = time.perf_counter()
    save_info = run_cli(["save", *common, "--dist-port", str(port + 17)])["save"]
    save_wall = time.perf_counter() - t0
    # 2) LOAD in a fresh process: cold start (spawn -> first token) and restore time.
    cold = {}
    if not args.skip_cold_start:
        cold = run_cli(["load", *common, "--dist-port", str(port + 19)],
                       {"FOUNDRY_SPAWN_T0_NS": str(time.time_ns())})["load"]

    # 3) This process restores the archive and runs the timed decode.
    from foundry_b200 import ops
    from foundry_b200.runner import persist

    eng, restore = persist.load(archive)
    cfg = eng.ecfg.model
    g = torch.Generator().manual_seed(1234 + (0 if mode == "tp" else rank))
    prompts = torch.randint(0, cfg.vocab, (args.batch, args.prompt_len), generator=g).tolist()
    reqs = eng.add_requests(prompts, max_new_tokens=gen)
    torch.cuda.synchronize()
    tp0 = time.perf_counter()
    eng.prefill(reqs)
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - tp0
    b = eng.start_decode(reqs)
    graph = eng.graphs[b]
    st = eng.state
    kernels_per_step = len(graph.desc.kernel_names())

    for _ in range(args.warmup):
        eng.decode_step(b)
    eng.wait_materialized()  # restored graphs get their own executables after the first step
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    sampler = ClockSampler(local)
    sampler.start()
    # Device-timed: K restored-graph steps back to back, sampled tokens fed back
    # on the device (one copy kernel per step), no host round trip.
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    for _ in range(args.steps):
        graph.replay()
        ops.copy_i32(st.next_ids[:b], st.input_ids[:b])
    end.record()
    torch.cuda.synchronize()
    dev_ms = start.elapsed_time(end)
    # Re-sync the host copy of the last tokens for the e2e phase.
    eng.h_in[:b].copy_(st.input_ids[:b])
    if world > 1:
        dist.barrier()
    # End to end through the public API: H2D inputs, graph launch, D2H tokens, sync.
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e_start.record()
    for _ in range(args.steps):
        eng.decode_step(b)
    e_end.record()
    torch.cuda.synchronize()
    e2e_ms = e_start.elapsed_time(e_end)
    clocks = sampler.stop()

    n_active = len(reqs)
    t = torch.tensor([dev_ms, e2e_ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
    dev_ms, e2e_ms = t.tolist()
    seq_ranks = 1 if mode == "tp" else world  # tp ranks share one batch of sequences
    tokens = n_active * seq_ranks * args.steps
    value = tokens / (dev_ms / 1e3)
    e2e = tokens / (e2e_ms / 1e3)
    if rank == 0:
        out = {
            "metric": f"restored decode tok/s ({args.model} shape, {restore['num_graphs']} persisted decode graphs)",
            "value": round(value, 1),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(dev_ms / args.steps, 4),
            "higher_is_better": True,
            "scaling": "strong" if mode == "tp" else "weak",
            "vs_baseline": None,
            "dtype": "fp8-block (e4m3, 128x128 fp32 scales) + bf16" if "qwen3" in args.model else "bf16",
            "data": "synthetic (uniform random prompt token ids, random-init N(0,0.02) weights)",
            "config": {
                "model": args.model, "global_batch": n_active * seq_ranks, "seq_len": args.prompt_len + gen,
                "prompt_len": args.prompt_len, "gen_len": args.gen, "parallelism": f"{mode}{world}",
                "decode_batch_per_gpu": b, "graphs_per_rank": restore["num_graphs"],
                "topology_groups": restore["num_groups"],
                "l2": "inputs larger than L2 (all weights + the KV cache are read every step)",
            },
            "clocks": clocks,
            "e2e": {"value": round(e2e, 1), "unit": "tokens/s", "h2d_bytes_per_step": 4 * b,
                    "d2h_bytes_per_step": 4 * b, "ms_per_step": round(e2e_ms / args.steps, 4)},
            "gpu_launches": (kernels_per_step + 1) * args.steps,
            "persistence": {
                "capture_s_67_graphs": save_info.get("capture_s"), "save_s": save_info.get("save_s"),
                "save_process_wall_s": round(save_wall, 2),
                "restore_s": round(restore["restore_s"], 4),
                "restore_phase1_ms": restore["restore_phase1_ms"],
                "restore_phase2_ms": restore["restore_phase2_ms"],
                "restore_s_per_256_graphs": round(restore["restore_s"] * 256 / restore["num_graphs"], 4),
                "cold_start_first_token_s": cold.get("cold_start_first_token_s"),
                "cold_start_restore_s": cold.get("restore_s"),
                "cold_start_breakdown_s": {k: cold.get(k) for k in ("python_import_s", "modules_s", "arena_s",
                                                                    "restore_s", "load_total_s")},
                "prefill_s": round(prefill_s, 3),
            },
        }
        print(json.dumps(out))
    eng.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
