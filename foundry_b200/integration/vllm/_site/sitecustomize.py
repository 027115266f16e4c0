"""Installs the foundry vLLM hooks at interpreter start in every process of a
vLLM engine (engine core and workers are spawned), when FOUNDRY_GRAPH_CONFIG
names a graph-extension TOML file. Put this folder on PYTHONPATH (the
``foundry_b200.integration.vllm.serve`` launcher does)."""

import os

if os.environ.get("FOUNDRY_GRAPH_CONFIG"):
    try:
        from foundry_b200.integration.vllm.hooks import install_hooks

        install_hooks(os.environ["FOUNDRY_GRAPH_CONFIG"])
    except ImportError:  # vLLM is not importable in this process (e.g. a helper)
        pass
