"""End-to-end check of the vLLM integration on one GPU: SAVE, then a fresh LOAD.

    python -m foundry_b200.integration.vllm.check --model llama-3-8b@2l --workdir /tmp/vllm_check

Runs upstream vLLM (offline ``LLM`` API, dummy weights from a local
``config.json``, token-id prompts, no tokenizer) twice, each in a fresh
process with the driver interposer preloaded and the engine core in-process
(``VLLM_ENABLE_V1_MULTIPROCESSING=0``):

1. SAVE, twice: vLLM captures its decode CUDA graphs (FULL_DECODE_ONLY)
   through the foundry hooks, which write them, the graph manifest and the
   packed modules into ``<workdir>/archive/rank_0``. The first pass also
   profiles memory and records the KV-cache budget; the second reuses it
   without profiling, so it allocates exactly as LOAD will;
2. LOAD: the same engine start restores the graphs instead of capturing them.

Both generate greedy tokens for the same prompts. Prints one JSON line with
the tokens' agreement, the number of graphs restored and their topology
groups, the restore time and each process's start-to-first-token time.

Parity: the manual SAVE -> LOAD -> compare workflow of the reference's vLLM
docs (docs/vllm/save-load-workflow.md:61-84).
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(os.path.dirname(HERE)))


def _toml(path: str, mode: str, workspace: str, base: str, region: str) -> str:
    with open(path, "w") as f:
        f.write(f'mode = "{mode}"\nbase_addr = "{base}"\nregion_size = "{region}"\n'
                f'workspace_root = "{workspace}"\nscratch_space_size = "512MB"\n')
    return path


def child(a) -> int:
    """One engine start (SAVE or LOAD) in this process; prints a JSON line."""
    t_start_ns = int(os.environ.get("FOUNDRY_SPAWN_T0_NS", time.time_ns()))
    from foundry_b200.integration import runtime
    from foundry_b200.integration.vllm.hooks import install_hooks

    install_hooks(a.config)
    import torch
    from vllm import LLM, SamplingParams

    sizes = [int(x) for x in a.sizes.split(",")]
    t0 = time.perf_counter()
    llm = LLM(model=a.model_dir, load_format="dummy", skip_tokenizer_init=True, dtype="bfloat16", seed=0,
              max_model_len=a.prompt_len + a.gen + 16, max_num_seqs=max(sizes), gpu_memory_utilization=a.mem,
              compilation_config={"cudagraph_mode": "FULL_DECODE_ONLY", "cudagraph_capture_sizes": sizes})
    engine_s = time.perf_counter() - t0
    g = torch.Generator().manual_seed(7)
    vocab = int(json.load(open(os.path.join(a.model_dir, "config.json")))["vocab_size"])
    prompts = [{"prompt_token_ids": torch.randint(3, vocab, (a.prompt_len,), generator=g).tolist()}
               for _ in range(a.prompts)]
    sp1 = SamplingParams(max_tokens=1, temperature=0.0, ignore_eos=True, detokenize=False)
    llm.generate(prompts[:1], sp1, use_tqdm=False)
    first_token_s = (time.time_ns() - t_start_ns) / 1e9
    sp = SamplingParams(max_tokens=a.gen, temperature=0.0, ignore_eos=True, detokenize=False)
    torch.cuda.synchronize()
    t = time.perf_counter()
    outs = llm.generate(prompts, sp, use_tqdm=False)
    torch.cuda.synchronize()
    gen_s = time.perf_counter() - t
    st = runtime.state()
    info = {"mode": a.mode, "tokens": [list(o.outputs[0].token_ids) for o in outs], "engine_init_s": engine_s,
            "start_to_first_token_s": first_token_s, "generate_s": gen_s}
    if st is not None and st.pending is not None and st.pending.pending is not None:
        p = st.pending.pending
        info.update({"graphs_restored": len(st.loaded), "graphs_in_archive": p.num_graphs,
                     "topology_groups": p.num_groups, "restore_phase1_ms": p.phase1_ms,
                     "restore_phase2_ms": p.phase2_ms})
    if st is not None:
        info["graphs_saved"] = st.capture_index
    print("FOUNDRY_CHECK " + json.dumps(info), flush=True)
    return 0


def run_child(mode: str, a, cfg_path: str, env_base: dict) -> dict:
    from foundry_b200.integration.config import GraphExtensionConfig
    from foundry_b200.integration.runtime import ld_preload_env

    env = ld_preload_env(env_base, GraphExtensionConfig.from_toml(cfg_path))
    env.update({"VLLM_ENABLE_V1_MULTIPROCESSING": "0", "NCCL_CUMEM_ENABLE": "0", "NCCL_NVLS_ENABLE": "0",
                "TORCH_CUBLASLT_UNIFIED_WORKSPACE": "1", "FOUNDRY_SPAWN_T0_NS": str(time.time_ns()),
                "PYTHONPATH": os.pathsep.join([ROOT, env_base.get("PYTHONPATH", "")])})
    cmd = [sys.executable, "-m", "foundry_b200.integration.vllm.check", "--child", mode, "--config", cfg_path,
           "--model-dir", a.model_dir, "--sizes", a.sizes, "--prompts", str(a.prompts), "--prompt-len",
           str(a.prompt_len), "--gen", str(a.gen), "--mem", str(a.mem)]
    t = time.perf_counter()
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=a.timeout)
    wall = time.perf_counter() - t
    with open(os.path.join(a.workdir, f"{mode}.log"), "w") as f:
        f.write(r.stdout + "\n---- stderr ----\n" + r.stderr)
    for line in r.stdout.splitlines():
        if line.startswith("FOUNDRY_CHECK "):
            info = json.loads(line[len("FOUNDRY_CHECK "):])
            info["process_wall_s"] = wall
            return info
    raise RuntimeError(f"{mode} run failed (rc {r.returncode}); log: {a.workdir}/{mode}.log\n{r.stderr[-3000:]}")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="foundry_b200.integration.vllm.check")
    ap.add_argument("--model", default="llama-3-8b@2l")
    ap.add_argument("--workdir", default="/tmp/foundry_vllm_check")
    ap.add_argument("--sizes", default="1,2,4,8")
    ap.add_argument("--prompts", type=int, default=8)
    ap.add_argument("--prompt-len", type=int, default=64)
    ap.add_argument("--gen", type=int, default=16)
    ap.add_argument("--mem", type=float, default=0.5, help="vLLM gpu_memory_utilization")
    ap.add_argument("--base-addr", default="0x600000000000")
    ap.add_argument("--region-size", default="120GB")
    ap.add_argument("--timeout", type=int, default=1200)
    ap.add_argument("--child", choices=["save", "load"])
    ap.add_argument("--config")
    ap.add_argument("--model-dir")
    a = ap.parse_args(argv)
    if a.child:
        a.mode = a.child
        return child(a)
    from foundry_b200.runner.vllm_baseline import write_model_dir

    os.makedirs(a.workdir, exist_ok=True)
    a.model_dir = write_model_dir(a.model, os.path.join(a.workdir, "model"))
    archive = os.path.join(a.workdir, "archive")
    save_cfg = _toml(os.path.join(a.workdir, "save.toml"), "save", archive, a.base_addr, a.region_size)
    save1 = run_child("save", a, save_cfg, dict(os.environ))
    os.replace(os.path.join(a.workdir, "save.log"), os.path.join(a.workdir, "save1.log"))
    save = run_child("save", a, save_cfg, dict(os.environ))
    load = run_child("load", a, _toml(os.path.join(a.workdir, "load.toml"), "load", archive, a.base_addr,
                                      a.region_size), dict(os.environ))
    out = {"model": a.model, "sizes": a.sizes, "tokens_match": save["tokens"] == load["tokens"],
           "save_passes_match": save1["tokens"] == save["tokens"],
           "graphs_saved": save.get("graphs_saved"), "graphs_restored": load.get("graphs_restored"),
           "graphs_in_archive": load.get("graphs_in_archive"), "topology_groups": load.get("topology_groups"),
           "restore_phase1_ms": load.get("restore_phase1_ms"), "restore_phase2_ms": load.get("restore_phase2_ms"),
           "save": {k: save[k] for k in ("engine_init_s", "start_to_first_token_s", "process_wall_s")},
           "load": {k: load[k] for k in ("engine_init_s", "start_to_first_token_s", "process_wall_s")}}
    print(json.dumps(out))
    return 0 if out["tokens_match"] else 1


if __name__ == "__main__":
    sys.exit(main())
