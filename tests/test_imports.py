"""Every public module and name imports on a CPU-only machine (the same guard
as the reference's tests/test_imports.py: re-exports must not go missing)."""

import importlib

import pytest

MODULES = [
    "foundry", "foundry_b200", "foundry_b200.allocation_region", "foundry_b200.graphs", "foundry_b200.ops",
    "foundry_b200.ops.gemm", "foundry_b200.ops.attention", "foundry_b200.ops.basic", "foundry_b200.ops.moe",
    "foundry_b200.models", "foundry_b200.models.llama", "foundry_b200.models.qwen3_moe", "foundry_b200.parallel.symm",
    "foundry_b200.parallel.comm", "foundry_b200.parallel.ep", "foundry_b200.runner.engine",
    "foundry_b200.runner.persist", "foundry_b200.runner.cli", "foundry_b200.runner.arena",
    "foundry_b200.runner.profile_gemm", "foundry_b200.runner.torch_baseline",
]

PUBLIC = [
    "CUDAGraph", "graph", "graph_pool_handle", "save_graph_manifest", "allocation_region", "parse_size",
    "set_allocation_region", "stop_allocation_region", "resume_allocation_region", "preallocate_region",
    "free_preallocated_region", "get_current_alloc_offset", "set_current_alloc_offset",
    "load_cuda_modules_and_libraries", "pack_fatbins_to_folder", "set_skip_fatbin_processing",
    "set_pack_fatbins_on_exit", "init_nvshmem_for_loaded_modules", "preallocate_cublas_workspaces",
]


@pytest.mark.parametrize("name", MODULES)
def test_module_imports(name):
    importlib.import_module(name)


def test_public_names():
    import foundry
    import foundry_b200

    for n in PUBLIC:
        assert hasattr(foundry_b200, n), n
        assert hasattr(foundry, n), n
    for n in ("start_graph_builds", "finish_graph_loads", "finish_one_graph_load", "load", "save"):
        assert hasattr(foundry.CUDAGraph, n), n
    # the extension-module names engine integrations use as `import foundry.ops as fops`
    import foundry.ops as fops

    for n in ("get_current_alloc_offset", "set_current_alloc_offset", "stop_allocation_region",
              "resume_allocation_region", "set_allocation_region", "preallocate_region", "preallocate_cublas_workspaces",
              "load_cuda_modules_and_libraries", "pack_fatbins_to_folder", "set_pack_fatbins_on_exit",
              "set_skip_fatbin_processing", "init_nvshmem_for_loaded_modules", "graph_pool_handle", "get_graph_ptr",
              "CUDAGraph"):
        assert hasattr(fops, n), n
    # reference module paths; the package attributes stay the context managers
    from foundry.allocation_region import parse_size
    from foundry.graph import save_graph_manifest
    import foundry.graph  # noqa: F401

    assert parse_size("1.5GB") == 3 << 29 and callable(save_graph_manifest)
    assert foundry.graph is foundry_b200.graph and foundry.allocation_region is foundry_b200.allocation_region


def test_model_configs():
    from foundry_b200.models import config_by_name, config_from_dict

    for name, params in (("llama-3-8b", 8.0e9), ("llama-3-70b", 70.5e9), ("qwen3-30b-a3b", 30.5e9)):
        cfg = config_by_name(name)
        assert abs(cfg.num_params() - params) / params < 0.03, (name, cfg.num_params())
        assert config_from_dict(cfg.to_dict()) == cfg
    c = config_by_name("qwen3-30b-a3b@2l")
    assert c.layers == 2 and c.num_experts == 128
