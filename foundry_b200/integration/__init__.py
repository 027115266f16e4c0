"""Engine integrations of the graph-persistence layer.

Engine-agnostic pieces: ``config`` (TOML graph-extension config, per-rank
workspaces), ``runtime`` (region setup, scratch skip, warm-up state, final
allocation offset, LD_PRELOAD environment) and ``graph_ops`` (archive file
naming, capture-or-load, LOAD pipeline, SAVE finalisation). Engine hooks:
``vllm`` (upstream vLLM V1), ``sglang``, ``trtllm`` (placeholder).
"""

from .config import GraphExtensionConfig, GraphExtensionMode, global_rank

__all__ = ["GraphExtensionConfig", "GraphExtensionMode", "global_rank"]
