"""Launch an SGLang server with the foundry graph extension in every process.

    python -m foundry_b200.integration.sglang.serve --foundry-config save.toml -- <sglang launch_server arguments>

Preloads the driver interposer (LD_PRELOAD), puts the sitecustomize shim on
PYTHONPATH with FOUNDRY_GRAPH_CONFIG and FOUNDRY_GRAPH_ENGINE=sglang (so every
SGLang process installs the SGLang hooks before it touches CUDA), turns
NCCL's cuMem / NVLS paths off (their allocations bypass the region), and
execs ``python -m sglang.launch_server``.
"""

from __future__ import annotations

import argparse
import os
import sys
import time

from ..config import GraphExtensionConfig
from ..runtime import ld_preload_env


def build_command(argv=None, environ=None) -> tuple[list[str], dict]:
    """(command, environment) of the launch; nothing is started."""
    ap = argparse.ArgumentParser(prog="foundry_b200.integration.sglang.serve")
    ap.add_argument("--foundry-config", required=True)
    ap.add_argument("rest", nargs=argparse.REMAINDER)
    a = ap.parse_args(argv)
    cfg = GraphExtensionConfig.from_toml(a.foundry_config)
    env = ld_preload_env(os.environ if environ is None else environ, cfg)
    site = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "vllm", "_site")
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    env["PYTHONPATH"] = os.pathsep.join([site, root] + [p for p in env.get("PYTHONPATH", "").split(os.pathsep) if p])
    env["FOUNDRY_GRAPH_CONFIG"] = os.path.abspath(a.foundry_config)
    env["FOUNDRY_GRAPH_ENGINE"] = "sglang"
    env["FOUNDRY_SPAWN_T0_NS"] = str(time.time_ns())
    env.setdefault("NCCL_CUMEM_ENABLE", "0")
    env.setdefault("NCCL_NVLS_ENABLE", "0")
    rest = [x for x in a.rest if x != "--"]
    return [sys.executable, "-m", "sglang.launch_server", *rest], env


def main(argv=None) -> int:
    cmd, env = build_command(argv)
    os.execvpe(cmd[0], cmd, env)
    return 0


if __name__ == "__main__":
    sys.exit(main())
