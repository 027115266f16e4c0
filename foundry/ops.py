"""``foundry.ops``: the module-level functions and the graph class under the
names the reference's extension module exports (python/foundry/ops.pyi:8-16,
used as ``import foundry.ops as fops`` by engine integrations), provided by
foundry_b200."""

from foundry_b200 import (  # noqa: F401
    CUDAGraph,
    free_preallocated_region,
    get_current_alloc_offset,
    graph_pool_handle,
    init_nvshmem_for_loaded_modules,
    load_cuda_modules_and_libraries,
    pack_fatbins_to_folder,
    preallocate_cublas_workspaces,
    preallocate_region,
    release_allocation_region,
    resume_allocation_region,
    set_allocation_region,
    set_current_alloc_offset,
    set_nvshmem_auto_init,
    set_pack_fatbins_on_exit,
    set_skip_fatbin_processing,
    stop_allocation_region,
)


def get_graph_ptr(graph: CUDAGraph) -> int:
    """The raw ``cudaGraph_t`` of a captured graph (0 if it has none)."""
    return int(graph.raw_cuda_graph() or 0)


__all__ = [
    "CUDAGraph", "free_preallocated_region", "get_current_alloc_offset", "get_graph_ptr", "graph_pool_handle",
    "init_nvshmem_for_loaded_modules", "load_cuda_modules_and_libraries", "pack_fatbins_to_folder",
    "preallocate_cublas_workspaces", "preallocate_region", "release_allocation_region", "resume_allocation_region",
    "set_allocation_region", "set_current_alloc_offset", "set_nvshmem_auto_init", "set_pack_fatbins_on_exit",
    "set_skip_fatbin_processing", "stop_allocation_region",
]
