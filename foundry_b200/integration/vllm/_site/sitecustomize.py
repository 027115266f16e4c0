"""Installs the foundry engine hooks at interpreter start in every process of
an engine (vLLM's engine core and workers, SGLang's schedulers are spawned),
when FOUNDRY_GRAPH_CONFIG names a graph-extension TOML file;
FOUNDRY_GRAPH_ENGINE selects the engine ("vllm", the default, or "sglang").
Put this folder on PYTHONPATH (the ``foundry_b200.integration.vllm.serve``
launcher does; the SGLang spawn-site patch exports both variables)."""

import os

if os.environ.get("FOUNDRY_GRAPH_CONFIG"):
    try:
        if os.environ.get("FOUNDRY_GRAPH_ENGINE", "vllm") == "sglang":
            from foundry_b200.integration.sglang.hooks import install_hooks
        else:
            from foundry_b200.integration.vllm.hooks import install_hooks

        install_hooks(os.environ["FOUNDRY_GRAPH_CONFIG"])
    except ImportError:  # the engine is not importable in this process (e.g. a helper)
        pass
