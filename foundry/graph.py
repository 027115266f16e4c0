"""``foundry.graph``: the graph capture / persistence names of the reference's
python/foundry/graph.py, provided by foundry_b200.graphs."""

from foundry_b200.graphs import CUDAGraph, graph, graph_pool_handle, save_graph_manifest  # noqa: F401

__all__ = ["CUDAGraph", "graph", "graph_pool_handle", "save_graph_manifest"]
