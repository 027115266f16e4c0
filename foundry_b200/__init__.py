"""foundry_b200: Blackwell-native CUDA-graph persistence framework.

Public API (same names as the reference's ``foundry`` package,
python/foundry/__init__.py:3-32 and ops.pyi):

* region: ``allocation_region``, ``parse_size``, ``set_allocation_region``,
  ``stop_allocation_region``, ``resume_allocation_region``,
  ``preallocate_region``, ``free_preallocated_region``,
  ``get_current_alloc_offset``, ``set_current_alloc_offset``
* graphs: ``CUDAGraph`` (capture / save / load / start_graph_builds /
  finish_graph_loads / finish_one_graph_load), ``graph``,
  ``save_graph_manifest``, ``graph_pool_handle``
* modules: ``pack_fatbins_to_folder``, ``load_cuda_modules_and_libraries``,
  ``set_skip_fatbin_processing``, ``set_pack_fatbins_on_exit``,
  ``set_nvshmem_auto_init``, ``init_nvshmem_for_loaded_modules``,
  ``preallocate_cublas_workspaces``, ``hook_library_path``
"""

from __future__ import annotations

from ._native import core, hook_library_path, use_mock_driver
from .allocation_region import (
    allocation_region,
    free_preallocated_region,
    get_current_alloc_offset,
    parse_size,
    preallocate_region,
    release_allocation_region,
    resume_allocation_region,
    set_allocation_region,
    set_current_alloc_offset,
    stop_allocation_region,
)

__version__ = "0.1.0"


def pack_fatbins_to_folder(folder_path: str) -> None:
    """Writes fatbin_image_packed.img + fatbin_entrypoint_packed.txt for every
    code image used by a saved graph."""
    core().pack_fatbins_to_folder(folder_path)


def load_cuda_modules_and_libraries(archive_dir: str) -> None:
    """Re-loads every image of an archive so saved graphs can resolve their kernels."""
    import torch

    if torch.cuda.is_available():
        torch.cuda.init()
    core().load_cuda_modules_and_libraries(archive_dir)


def set_skip_fatbin_processing(enabled: bool) -> None:
    core().set_skip_fatbin_processing(bool(enabled))


def set_pack_fatbins_on_exit(enabled: bool | str, folder: str | None = None) -> None:
    """Packs used images at process exit into ``folder`` (or a str argument)."""
    if isinstance(enabled, str):
        folder, enabled = enabled, True
    core().set_pack_fatbins_on_exit(folder if enabled and folder else None)


_nvshmem_auto_init = True


def set_nvshmem_auto_init(enabled: bool) -> None:
    """Kept for API parity. foundry_b200's kernels use their own symmetric memory
    (foundry_b200.parallel), never NVSHMEM, so there is nothing to initialise."""
    global _nvshmem_auto_init
    _nvshmem_auto_init = bool(enabled)


def init_nvshmem_for_loaded_modules() -> int:
    """API parity: returns the number of NVSHMEM-dependent modules initialised (always 0)."""
    return 0


def preallocate_cublas_workspaces() -> None:
    """Touches the cuBLAS/cuBLASLt handles of the current stream so their
    workspaces are allocated now, at a deterministic point of the cursor.
    (foundry_b200's own graphs use no cuBLAS; this serves user graphs that do.)"""
    import torch

    a = torch.zeros(16, 16, device="cuda", dtype=torch.float16)
    (a @ a).sum().item()


# Same names as the reference package: `graph` is the capture context manager
# (the implementation module is foundry_b200.graphs).
from .graphs import CUDAGraph, graph, graph_pool_handle, save_graph_manifest  # noqa: E402


__all__ = [
    "CUDAGraph", "allocation_region", "core", "free_preallocated_region", "get_current_alloc_offset", "graph",
    "graph_pool_handle", "hook_library_path", "init_nvshmem_for_loaded_modules", "load_cuda_modules_and_libraries",
    "pack_fatbins_to_folder", "parse_size", "preallocate_cublas_workspaces", "preallocate_region",
    "release_allocation_region", "resume_allocation_region", "save_graph_manifest", "set_allocation_region",
    "set_current_alloc_offset", "set_nvshmem_auto_init", "set_pack_fatbins_on_exit", "set_skip_fatbin_processing",
    "stop_allocation_region", "use_mock_driver",
]
