"""Launch ``vllm serve`` with the foundry graph extension in every engine process.

    python -m foundry_b200.integration.vllm.serve --foundry-config save.toml -- <vllm serve arguments>

Sets FOUNDRY_GRAPH_CONFIG, puts the sitecustomize shim on PYTHONPATH, preloads
the driver interposer (LD_PRELOAD) and execs vLLM's CLI, so the engine core
and its workers install the hooks before they touch CUDA. vLLM should run with
FULL_DECODE_ONLY (or FULL) CUDA graphs; NCCL's cuMem / NVLS paths are turned
off because their allocations bypass the region (NCCL_CUMEM_ENABLE=0,
NCCL_NVLS_ENABLE=0), as in the reference recipes (recipe/vllm/README.md:165-189).
"""

from __future__ import annotations

import argparse
import os
import shutil
import sys
import time

from ..config import GraphExtensionConfig
from ..runtime import ld_preload_env


def build_command(argv=None, environ=None) -> tuple[list[str], dict]:
    """(command, environment) of the launch; nothing is started."""
    ap = argparse.ArgumentParser(prog="foundry_b200.integration.vllm.serve")
    ap.add_argument("--foundry-config", required=True)
    ap.add_argument("rest", nargs=argparse.REMAINDER)
    a = ap.parse_args(argv)
    cfg = GraphExtensionConfig.from_toml(a.foundry_config)
    env = ld_preload_env(os.environ if environ is None else environ, cfg)
    site = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_site")
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    env["PYTHONPATH"] = os.pathsep.join([site, root] + [p for p in env.get("PYTHONPATH", "").split(os.pathsep) if p])
    env["FOUNDRY_GRAPH_CONFIG"] = os.path.abspath(a.foundry_config)
    env["FOUNDRY_SPAWN_T0_NS"] = str(time.time_ns())  # engine processes log their start-up cost from here
    env.setdefault("NCCL_CUMEM_ENABLE", "0")
    env.setdefault("NCCL_NVLS_ENABLE", "0")
    rest = [x for x in a.rest if x != "--"]
    vllm = shutil.which("vllm")
    cmd = [vllm, "serve", *rest] if vllm else [sys.executable, "-m", "vllm.entrypoints.cli.main", "serve", *rest]
    return cmd, env


def main(argv=None) -> int:
    cmd, env = build_command(argv)
    os.execvpe(cmd[0], cmd, env)
    return 0


if __name__ == "__main__":
    sys.exit(main())
