"""Headline benchmark: restored-graph decode throughput of the Llama-3-8B-shaped
serving load (256 prompts x 512 random tokens, greedy) on N GPUs (DP: one
full engine per GPU, weak scaling), plus the persistence numbers of the same
run: graph capture + SAVE, fresh-process cold start to first token, and
restore time of the 67 decode graphs, and a second SAVE / fresh-process
LOAD of 256 decode graphs per rank (restore time measured, not scaled).

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

REF_DIR = os.path.join(ROOT, "baseline", "_ref")
REF_INSTALL_FAILURE = (
    "the offline install (pip install --no-index --no-deps --target baseline/_ref <reference copy>) fails at the "
    "reference's CMake configure step: CMakeLists.txt:9 find_package(Boost) finds no Boost>=1.83 on this image "
    "and there is no network"
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
    ap.add_argument("--skip-full-generation", action="store_true",
                    help="leave out the timed whole generation after the decode window (its second prefill)")
    ap.add_argument("--restore-graphs", default="4:1024:4",
                    help="graph sizes of the restore-at-scale SAVE/LOAD (default: 256 graphs); 'none' skips it")
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


def replica_visibility(local: int, environ) -> tuple[dict, int]:
    """(environment, device ordinal) for a data-parallel replica's SAVE / LOAD
    processes: only the replica's own GPU visible (``local`` indexes the
    launcher's CUDA_VISIBLE_DEVICES list when it has one), as device 0."""
    vis = environ.get("CUDA_VISIBLE_DEVICES")
    ids = [v.strip() for v in vis.split(",") if v.strip()] if vis else []
    return {"CUDA_VISIBLE_DEVICES": ids[local] if local < len(ids) else str(local)}, 0


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


def run_reference(rank: int) -> int:
    """The reference arm: imports the reference's own package from
    baseline/_ref in a clean interpreter (this repository's ``foundry`` alias
    package must not shadow it). The reference persists graphs of the vLLM /
    SGLang forks it patches, neither of which is on the image, so even an
    importable build would have no engine to serve the benchmark; the import
    is still tried so that the reason printed is the one observed."""
    reason = None
    if not os.path.isdir(REF_DIR):
        reason = f"baseline/_ref is absent: {REF_INSTALL_FAILURE}"
    else:
        res = subprocess.run([sys.executable, "-c", "import foundry, foundry.ops; print(foundry.__file__)"],
                             cwd="/tmp", env={**{k: v for k, v in os.environ.items() if k != "PYTHONPATH"},
                                              "PYTHONPATH": REF_DIR},
                             capture_output=True, text=True, timeout=300)
        if res.returncode != 0:
            err = (res.stderr.strip().splitlines() or ["no output"])[-1]
            reason = f"importing the reference from baseline/_ref failed: {err}"
        else:
            reason = ("the reference imports, but its decode path is the foundry-org vLLM/SGLang forks, which are "
                      "not on the image; upstream vLLM 0.22 lacks the graph-extension hooks it patches")
    if rank == 0:
        print(json.dumps({"impl": "reference", "unavailable": reason}))
    return 0


def main():
    args = parse()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        return run_reference(rank)

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
    # A data-parallel replica needs no other GPU: its SAVE / LOAD processes see
    # only their own device, so CUDA initialises one device instead of every
    # GPU of the node (with eight ranks starting at once, context creation was
    # most of the time to first token). TP / EP ranks map peers' memory and see
    # all devices.
    child_env, child_dev = ({}, local) if mode != "dp" else replica_visibility(local, os.environ)
    common = ["--archive", archive, "--model", args.model, "--prompts", str(args.batch), "--prompt-len",
              str(args.prompt_len), "--gen", str(gen), "--device", str(child_dev), "--graph-sizes", args.graph_sizes,
              "--region-size", args.region_size]
    if mode in ("tp", "ep"):
        common += [f"--{mode}", str(world), "--rank", str(rank), "--world", str(world)]

    # 1) SAVE in a fresh process: capture the decode graphs and write the archive.
    t0 = time.perf_counter()
    save_info = run_cli(["save", *common, "--dist-port", str(port + 17)], child_env)["save"]
    save_wall = time.perf_counter() - t0
    # 2) LOAD in a fresh process: cold start (spawn -> first token) and restore time.
    cold = {}
    if not args.skip_cold_start:
        cold = run_cli(["load", *common, "--dist-port", str(port + 19)],
                       dict(child_env, FOUNDRY_SPAWN_T0_NS=str(time.time_ns()),
                            FOUNDRY_EARLY_CUDA_INIT=str(child_dev)))["load"]

    # 2b) Restore at scale: a second archive of 256 decode graphs per rank,
    # SAVE and fresh-process LOAD; the LOAD times until every graph of the
    # archive also has its own executable (the cost if each graph were its own
    # topology group).
    scale = {}
    if args.restore_graphs != "none":
        archive256 = os.path.join(workdir, f"scale_rank_{rank}") if mode == "dp" else workdir + "_scale"
        common256 = list(common)
        common256[common256.index("--archive") + 1] = archive256
        common256[common256.index("--graph-sizes") + 1] = args.restore_graphs
        save256 = run_cli(["save", *common256, "--dist-port", str(port + 23)], child_env)["save"]
        load256 = run_cli(["load", *common256, "--dist-port", str(port + 29), "--materialize-all"],
                          dict(child_env, FOUNDRY_SPAWN_T0_NS=str(time.time_ns()),
                               FOUNDRY_EARLY_CUDA_INIT=str(child_dev)))["load"]
        scale = {"graphs": load256["num_graphs"], "topology_groups": load256["num_groups"],
                 "capture_s": save256.get("capture_s"), "restore_s": load256["restore_s"],
                 "cold_start_first_token_s": load256["cold_start_first_token_s"],
                 "materialize_all_s_after_first_token": load256.get("materialize_all_s_after_first_token")}

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

    ctx0 = args.prompt_len + 1  # tokens in the cache at the first decode step
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
    dev_ctx = [ctx0 + args.warmup, ctx0 + args.warmup + args.steps - 1]
    e2e_ctx = [dev_ctx[1] + 1, dev_ctx[1] + args.steps]

    # Whole serving load through the public API: fresh requests, prefill, then
    # every decode step of the args.gen-token generation (context prompt_len+1
    # .. prompt_len+gen-1), each with its H2D input and D2H token copy.
    n_full = len(reqs)
    eng.release(reqs)
    full_ms, fb = 0.0, b
    if not args.skip_full_generation:
        freqs = eng.add_requests(prompts, max_new_tokens=args.gen)
        eng.prefill(freqs)
        fb = eng.start_decode(freqs)
        if world > 1:
            dist.barrier()
        f_start, f_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        f_start.record()
        for _ in range(args.gen - 1):
            eng.decode_step(fb)
        f_end.record()
        torch.cuda.synchronize()
        full_ms = f_start.elapsed_time(f_end)
        eng.release(freqs)

    n_active = n_full
    per_rank = [dev_ms, e2e_ms, full_ms, restore["restore_s"], cold.get("cold_start_first_token_s") or 0.0,
                scale.get("restore_s") or 0.0, scale.get("cold_start_first_token_s") or 0.0,
                scale.get("materialize_all_s_after_first_token") or 0.0]
    t = torch.tensor(per_rank, dtype=torch.float64, device="cuda")
    if world > 1:  # every time below is the maximum over ranks
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
    (dev_ms, e2e_ms, full_ms, restore_max, cold_max, scale_restore_max, scale_cold_max,
     scale_mat_max) = t.tolist()
    seq_ranks = 1 if mode == "tp" else world  # tp ranks share one batch of sequences
    tokens = n_active * seq_ranks * args.steps
    value = tokens / (dev_ms / 1e3)
    e2e = tokens / (e2e_ms / 1e3)
    full_tokens = n_active * seq_ranks * (args.gen - 1)
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
                "decode_context_timed": dev_ctx, "decode_context_e2e": e2e_ctx,
                "l2": "inputs larger than L2 (all weights + the KV cache are read every step)",
            },
            "clocks": clocks,
            "e2e": {"value": round(e2e, 1), "unit": "tokens/s", "h2d_bytes_per_step": 4 * b,
                    "d2h_bytes_per_step": 4 * b, "ms_per_step": round(e2e_ms / args.steps, 4),
                    "decode_context": e2e_ctx},
            "full_generation": None if args.skip_full_generation else {
                "value": round(full_tokens / (full_ms / 1e3), 1), "unit": "tokens/s",
                "decode_steps": args.gen - 1, "decode_context": [ctx0, args.prompt_len + args.gen - 1],
                "ms_per_step": round(full_ms / (args.gen - 1), 4), "h2d_bytes_per_step": 4 * fb,
                "d2h_bytes_per_step": 4 * fb,
                "how": "public API decode_step for every step of the generation after prefill, CUDA events, "
                       "max over ranks"},
            "gpu_launches": (kernels_per_step + 1) * args.steps,
            "persistence": {
                "capture_s": save_info.get("capture_s"), "captured_graphs": restore["num_graphs"],
                "save_s": save_info.get("save_s"),
                "save_process_wall_s": round(save_wall, 2),
                "restore_s": round(restore_max, 4),
                "restore_phase1_ms": restore["restore_phase1_ms"],
                "restore_phase2_ms": restore["restore_phase2_ms"],
                "cold_start_first_token_s": round(cold_max, 3) if cold else None,
                "cold_start_restore_s": cold.get("restore_s"),
                "cold_start_breakdown_s": {k: cold.get(k) for k in ("python_import_s", "modules_s", "arena_s",
                                                                    "restore_s", "load_total_s",
                                                                    "cold_start_steps_s", "early_cuda_context")},
                "prefill_s": round(prefill_s, 3),
                "restore_at_scale": dict(scale, restore_s=round(scale_restore_max, 4),
                                         cold_start_first_token_s=round(scale_cold_max, 3),
                                         materialize_all_s_after_first_token=round(scale_mat_max, 3),
                                         ranks=world, how="max over ranks; fresh-process LOAD of a "
                                                           "separately saved archive") if scale else None,
                "times": "max over ranks",
            },
        }
        print(json.dumps(out))
    eng.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
