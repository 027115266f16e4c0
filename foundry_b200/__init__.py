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

from . import _early_cuda

# Before anything imports torch: build the CUDA context meanwhile, if asked.
_early_cuda.start_from_env()

from ._native import core, hook_library_path, use_mock_driver  # noqa: E402
from .allocation_region import (  # noqa: E402
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
    """Re-loads every image of an archive so saved graphs can resolve their
    kernels. Images that need NVSHMEM are queued for
    ``init_nvshmem_for_loaded_modules``; with auto-init on (the default) they
    are initialised right away when the process has already loaded an NVSHMEM
    host library, and otherwise stay queued."""
    import torch

    if torch.cuda.is_available():
        torch.cuda.init()
    core().load_cuda_modules_and_libraries(archive_dir)
    if _nvshmem_auto_init:
        try:
            core().init_nvshmem_modules()
        except RuntimeError:
            pass  # NVSHMEM not up yet: init_nvshmem_for_loaded_modules() after its bootstrap


def set_skip_fatbin_processing(enabled: bool) -> None:
    core().set_skip_fatbin_processing(bool(enabled))


def set_pack_fatbins_on_exit(enabled: bool | str, folder: str | None = None) -> None:
    """Packs used images at process exit into ``folder`` (or a str argument)."""
    if isinstance(enabled, str):
        folder, enabled = enabled, True
    core().set_pack_fatbins_on_exit(folder if enabled and folder else None)


_nvshmem_auto_init = True


def set_nvshmem_auto_init(enabled: bool) -> None:
    """Whether ``load_cuda_modules_and_libraries`` tries to initialise
    NVSHMEM-dependent images itself (foundry_b200's own kernels use their own
    symmetric memory and never need it; images of libraries such as DeepEP do)."""
    global _nvshmem_auto_init
    _nvshmem_auto_init = bool(enabled)


def init_nvshmem_for_loaded_modules() -> int:
    """Initialises every reloaded image that needs NVSHMEM with the process's
    NVSHMEM host library (``nvshmemx_cumodule_init`` /
    ``nvshmemx_culibrary_init``, looked up in the process, never loaded here);
    call it after the NVSHMEM runtime is bootstrapped. Returns how many images
    were initialised (0 when none was pending); raises RuntimeError when some
    are pending but no NVSHMEM host library is loaded, or an init fails.
    Parity: reference csrc/hook.cpp:1193-1365."""
    return core().init_nvshmem_modules()


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
from . import jit as _jit  # noqa: E402

# Kernels Triton compiles in this process (torch.compile / Inductor) are
# adopted by the registry as they load, so graphs that use them persist.
_jit.install()


__all__ = [
    "CUDAGraph", "allocation_region", "core", "free_preallocated_region", "get_current_alloc_offset", "graph",
    "graph_pool_handle", "hook_library_path", "init_nvshmem_for_loaded_modules", "load_cuda_modules_and_libraries",
    "pack_fatbins_to_folder", "parse_size", "preallocate_cublas_workspaces", "preallocate_region",
    "release_allocation_region", "resume_allocation_region", "save_graph_manifest", "set_allocation_region",
    "set_current_alloc_offset", "set_nvshmem_auto_init", "set_pack_fatbins_on_exit", "set_skip_fatbin_processing",
    "stop_allocation_region", "use_mock_driver",
]
