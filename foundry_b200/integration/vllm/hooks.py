"""vLLM (V1 engine, 0.22) integration: persist the engine's CUDA graphs.

``install_hooks(config)`` patches, in the current process:

  CUDAGraphWrapper.__call__        capture -> foundry capture + save (SAVE) or
                                   restore (LOAD) keyed by the batch descriptor
  init_worker_distributed_environment  (first step of Worker.init_device)
                                   right after the communicator is up: LOAD
                                   loads the packed modules, both modes enable
                                   the region and skip the scratch space, before
                                   the workspace manager and the model runner's
                                   persistent buffers are allocated
  Worker.determine_available_memory  the first SAVE pass profiles and records
                                   the KV-cache budget; a second SAVE pass and
                                   LOAD reuse it without profiling, so they
                                   allocate identically (save twice, then load)
  GPUModelRunner.initialize_kv_cache SAVE records the KV-cache addresses, LOAD
                                   checks them before any graph is restored
  kernel_warmup (gpu_worker)       skipped in SAVE and LOAD (it allocates)
  GPUModelRunner.load_model        LOAD: map SAVE's working set in one piece
                                   before the weights load, start the graph
                                   builds right after (they overlap the KV
                                   cache setup and profiling that follow)
  GPUModelRunner._dummy_run        SAVE/LOAD: the one eager sampler-warm-up
                                   forward (runtime mode NONE, skip_eplb, no
                                   profile/capture/attention/decode flag)
                                   returns zero hidden states instead of
                                   running the model; every other dummy run
                                   (profiling, capture, DP padding) runs
  GPUModelRunner.capture_model     LOAD: start all graph builds first (if not
                                   already), afterwards give every restored
                                   graph its own executable on a background
                                   thread; SAVE: manifest + packed modules +
                                   final offset
  prepare_communication_buffer_for_model  LOAD: initialise the reloaded
                                   images that need NVSHMEM once DeepEP has
                                   bootstrapped it (when the target exists)
  DeepEPLLAll2AllManager._make_all2all_kwargs  fabric-handle buffers, no
                                   NVLink buffer (when DeepEP is present)
  torch.cuda.get_device_capability answered from NVML, so importing a kernel
                                   library in the API-server process does not
                                   create a CUDA context there (a process that
                                   has one cannot fork engine workers)

Spawned engine processes install the same hooks through the
``_site/sitecustomize.py`` shim when FOUNDRY_GRAPH_CONFIG names the TOML file
(``python -m foundry_b200.integration.vllm.serve`` sets it up).

Parity: reference python/foundry/integration/vllm/hooks.py:85-706 (10 patches
against foundry-org's vLLM fork); these target upstream vLLM.
"""

from __future__ import annotations

import logging
import os
import time

from .. import graph_ops, runtime
from ..config import GraphExtensionConfig, GraphExtensionMode, global_rank

log = logging.getLogger("foundry")

_originals: dict = {}


def _targets():
    import vllm.compilation.cuda_graph as cg
    import vllm.v1.worker.gpu_model_runner as mr
    import vllm.v1.worker.gpu_worker as gw

    return cg, gw, mr


def _wrapper_call(self, *args, **kwargs):
    from vllm.compilation.cuda_graph import CUDAGraphEntry
    from vllm.config import CUDAGraphMode
    from vllm.forward_context import get_forward_context, is_forward_context_available

    if runtime.mode() == GraphExtensionMode.NONE:
        return _originals["CUDAGraphWrapper.__call__"](self, *args, **kwargs)
    if not is_forward_context_available():
        return self.runnable(*args, **kwargs)
    fc = get_forward_context()
    bd, rm = fc.batch_descriptor, fc.cudagraph_runtime_mode
    if rm == CUDAGraphMode.NONE or rm != self.runtime_mode:
        return self.runnable(*args, **kwargs)
    entry = self.concrete_cudagraph_entries.get(bd)
    if entry is None:
        entry = self.concrete_cudagraph_entries[bd] = CUDAGraphEntry(batch_descriptor=bd)
    if entry.cudagraph is None:
        pc = getattr(self.runnable, "piecewise_compile_index", None) if rm == CUDAGraphMode.PIECEWISE else None
        key = graph_ops.GraphKey(rm.name, bd.num_tokens, bd.num_reqs, bool(bd.uniform), bool(bd.has_lora), pc)
        import torch

        g, out = graph_ops.capture_or_load(key, self.runnable, args, kwargs, pool=self.graph_pool,
                                           stream=torch.cuda.current_stream())
        entry.cudagraph = g
        entry.output = out
        return out
    entry.cudagraph.replay()
    return entry.output


def _init_distributed(vllm_config, rank, *a, **k):
    """Worker.init_device calls this first; the workspace manager and the model
    runner's persistent input buffers are allocated right after it, so the
    region (and, on LOAD, the packed modules) is set up as soon as the
    communicator is up, before any of those allocations."""
    r = _originals["init_worker_distributed_environment"](vllm_config, rank, *a, **k)
    cfg = _config
    pc = vllm_config.parallel_config
    grank = global_rank(rank, pc.world_size, getattr(pc, "data_parallel_rank", 0) or 0)
    runtime.setup_graph_extension(cfg, grank)
    if cfg.mode != GraphExtensionMode.NONE:
        runtime.skip_to_scratch_boundary()
    return r


def _determine_available_memory(self, *a, **k):
    """KV-cache budget. The first SAVE pass measures it (vLLM's profiling
    allocates and captures graphs of its own) and records it; a second SAVE
    pass and every LOAD reuse it without profiling, so they allocate the
    same buffers in the same order and the KV cache lands at the same
    address. Parity: reference vllm/hooks.py:536-642."""
    st = runtime.state()
    if st is None or st.config.mode == GraphExtensionMode.NONE:
        return _originals["Worker.determine_available_memory"](self, *a, **k)
    ws = st.config.workspace_dir
    saved = runtime.WarmupState.load(ws)
    if saved is not None and "available_memory" in saved.extra:
        return int(saved.extra["available_memory"])
    if st.config.mode == GraphExtensionMode.LOAD:
        raise RuntimeError(f"LOAD needs {ws}/warmup_state.json from a SAVE run")
    v = _originals["Worker.determine_available_memory"](self, *a, **k)
    runtime.WarmupState(extra={"available_memory": int(v)}).save(ws)
    log.info("[foundry] SAVE pass 1 recorded the KV-cache budget (%d bytes); run SAVE again for the "
             "deterministic pass that LOAD reproduces", int(v))
    return v


def _kv_cache_ptrs(runner) -> list[int]:
    out: list[int] = []

    def walk(x):
        if hasattr(x, "data_ptr"):
            out.append(int(x.data_ptr()))
        elif isinstance(x, (list, tuple)):
            for y in x:
                walk(y)
        elif isinstance(x, dict):
            for y in x.values():
                walk(y)

    walk(getattr(runner, "kv_caches", []))
    return out


def _initialize_kv_cache(self, *a, **k):
    """SAVE records the KV-cache tensors' addresses; LOAD checks them before
    any graph is restored (a restored graph reads the KV cache at SAVE's
    address, so a different layout must stop here, not in a kernel)."""
    r = _originals["GPUModelRunner.initialize_kv_cache"](self, *a, **k)
    st = runtime.state()
    if st is None or st.config.mode == GraphExtensionMode.NONE or k.get("is_profiling"):
        return r
    ptrs = _kv_cache_ptrs(self)
    ws = st.config.workspace_dir
    saved = runtime.WarmupState.load(ws) or runtime.WarmupState()
    if st.config.mode == GraphExtensionMode.SAVE:
        saved.extra["kv_cache_ptrs"] = ptrs
        saved.save(ws)
    elif saved.extra.get("kv_cache_ptrs") is not None and saved.extra["kv_cache_ptrs"] != ptrs:
        want = saved.extra["kv_cache_ptrs"]
        raise RuntimeError(f"LOAD placed the KV cache at {hex(ptrs[0]) if ptrs else None}, SAVE at "
                           f"{hex(want[0]) if want else None} ({len(ptrs)} vs {len(want)} tensors): this run "
                           "allocated differently before the KV cache (SAVE twice so the archive comes from the "
                           "deterministic second pass)")
    return r


def _kernel_warmup(worker, *a, **k):
    # Kernel warm-up (autotuning) allocates as it goes: skipped whenever graphs
    # are persisted, in SAVE as in LOAD (reference vllm/hooks.py:187-198).
    if runtime.mode() != GraphExtensionMode.NONE:
        return None
    return _originals["kernel_warmup"](worker, *a, **k)


def _load_model(self, *a, **k):
    st = runtime.state()
    if st is None or st.config.mode != GraphExtensionMode.LOAD:
        return _originals["GPUModelRunner.load_model"](self, *a, **k)
    t0 = time.perf_counter()
    runtime.preallocate_for_load_mode()
    r = _originals["GPUModelRunner.load_model"](self, *a, **k)
    graph_ops.start_graph_builds(st.config.workspace_dir)
    log.info("[foundry TIMING] load_model (preallocate + weights + start graph builds): %.3f s",
             time.perf_counter() - t0)
    return r


def is_sampler_warmup_run(kwargs: dict) -> bool:
    """The eager full forward vLLM runs once before the sampler warm-up
    (Worker.compile_or_warm_up_model): runtime mode NONE with skip_eplb and
    none of the flags that mark profiling, capture, forced attention or a
    uniform-decode (DP padding) batch."""
    mode = kwargs.get("cudagraph_runtime_mode")
    return (mode is not None and getattr(mode, "name", None) == "NONE" and kwargs.get("skip_eplb") is True
            and not any(kwargs.get(f) for f in ("is_profile", "is_graph_capturing", "force_attention",
                                                "uniform_decode")))


def _dummy_run(self, *a, **k):
    if runtime.mode() == GraphExtensionMode.NONE or not is_sampler_warmup_run(k):
        return _originals["GPUModelRunner._dummy_run"](self, *a, **k)
    import torch

    n = int(a[0]) if a else int(k.get("num_tokens", 1))
    hs = torch.zeros(n, self.model_config.get_hidden_size(), device=self.device, dtype=self.model_config.dtype)
    return hs, hs


def nvml_device_capability(device=None, _nvml=None) -> tuple[int, int]:
    """(major, minor) of ``device`` from NVML (no CUDA context is created)."""
    nv = _nvml
    if nv is None:
        import pynvml as nv
    if not _nvml_started.get(id(nv)):
        nv.nvmlInit()
        _nvml_started[id(nv)] = True
    if device is None:
        idx = 0
    elif isinstance(device, int):
        idx = device
    elif isinstance(device, str):
        idx = int(device.split(":")[-1]) if ":" in device else 0
    else:  # torch.device
        idx = device.index or 0
    major, minor = nv.nvmlDeviceGetCudaComputeCapability(nv.nvmlDeviceGetHandleByIndex(idx))
    return int(major), int(minor)


_nvml_started: dict = {}


def _quarantine_capability() -> None:
    import torch

    orig = torch.cuda.get_device_capability
    _originals["torch.cuda.get_device_capability"] = orig

    def capability(device=None):
        try:
            return nvml_device_capability(device)
        except Exception:
            return orig(device)

    torch.cuda.get_device_capability = capability


def _capture_model(self, *a, **k):
    st = runtime.state()
    if st is not None and st.config.mode == GraphExtensionMode.LOAD:
        graph_ops.start_graph_builds(st.config.workspace_dir)
    r = _originals["GPUModelRunner.capture_model"](self, *a, **k)
    if st is not None and st.config.mode == GraphExtensionMode.SAVE:
        graph_ops.finalize_save()
    if st is not None and st.config.mode != GraphExtensionMode.NONE:
        runtime.capture_final_alloc_offset()
    if st is not None and st.config.mode == GraphExtensionMode.LOAD:
        graph_ops.materialize_loaded(background=True)
    return r


def _prepare_comm_buffer(model, *a, **k):
    """After vLLM builds its communication buffers (DeepEP's Buffer bootstraps
    NVSHMEM there), LOAD initialises the reloaded images that need NVSHMEM;
    earlier, the NVSHMEM runtime is not up. Parity: reference
    vllm/hooks.py:350-374."""
    r = _originals["prepare_communication_buffer_for_model"](model, *a, **k)
    if runtime.mode() == GraphExtensionMode.LOAD:
        from ... import init_nvshmem_for_loaded_modules

        t = time.perf_counter()
        n = init_nvshmem_for_loaded_modules()
        log.info("[foundry TIMING] init_nvshmem_for_loaded_modules: %.3f s (%d images)", time.perf_counter() - t, n)
    return r


def _deepep_kwargs(self, *a, **k):
    """DeepEP low-latency buffers: fabric-handle memory (which the region
    sees and maps like its own) and no NVLink buffer, whenever graphs are
    persisted. Parity: reference vllm/hooks.py:682-706."""
    out = _originals["DeepEPLLAll2AllManager._make_all2all_kwargs"](self, *a, **k)
    if isinstance(out, dict) and runtime.mode() != GraphExtensionMode.NONE:
        out["use_fabric"] = True
        out["num_nvl_bytes"] = 0
    return out


def _optional_targets() -> list[tuple[str, object, str, object]]:
    """(key, owner, attribute, replacement) of patches whose targets vLLM
    builds may not have (absent targets are skipped)."""
    out = []
    import vllm.v1.worker.gpu_model_runner as mr

    if hasattr(mr, "prepare_communication_buffer_for_model"):
        out.append(("prepare_communication_buffer_for_model", mr, "prepare_communication_buffer_for_model",
                     _prepare_comm_buffer))
    try:
        from vllm.distributed.device_communicators import all2all
    except Exception:  # noqa: BLE001 - optional component
        all2all = None
    cls = getattr(all2all, "DeepEPLLAll2AllManager", None) if all2all is not None else None
    if cls is not None and hasattr(cls, "_make_all2all_kwargs"):
        out.append(("DeepEPLLAll2AllManager._make_all2all_kwargs", cls, "_make_all2all_kwargs", _deepep_kwargs))
    return out


_optional_installed: list[tuple[str, object, str]] = []
_config: GraphExtensionConfig | None = None


def install_hooks(config: GraphExtensionConfig | str) -> None:
    """Patches vLLM in this process (idempotent)."""
    global _config
    if isinstance(config, (str, os.PathLike)):
        config = GraphExtensionConfig.from_toml(config)
    _config = config
    if _originals:
        return
    t0 = os.environ.get("FOUNDRY_SPAWN_T0_NS")
    if t0:
        log.info("[foundry TIMING] process start -> install_hooks: %.1f ms", (time.time_ns() - int(t0)) / 1e6)
    _quarantine_capability()
    cg, gw, mr = _targets()
    _originals["CUDAGraphWrapper.__call__"] = cg.CUDAGraphWrapper.__call__
    _originals["init_worker_distributed_environment"] = gw.init_worker_distributed_environment
    _originals["Worker.determine_available_memory"] = gw.Worker.determine_available_memory
    _originals["kernel_warmup"] = gw.kernel_warmup
    _originals["GPUModelRunner.capture_model"] = mr.GPUModelRunner.capture_model
    _originals["GPUModelRunner.load_model"] = mr.GPUModelRunner.load_model
    _originals["GPUModelRunner._dummy_run"] = mr.GPUModelRunner._dummy_run
    _originals["GPUModelRunner.initialize_kv_cache"] = mr.GPUModelRunner.initialize_kv_cache
    cg.CUDAGraphWrapper.__call__ = _wrapper_call
    gw.init_worker_distributed_environment = _init_distributed
    gw.Worker.determine_available_memory = _determine_available_memory
    gw.kernel_warmup = _kernel_warmup
    mr.GPUModelRunner.capture_model = _capture_model
    mr.GPUModelRunner.load_model = _load_model
    mr.GPUModelRunner._dummy_run = _dummy_run
    mr.GPUModelRunner.initialize_kv_cache = _initialize_kv_cache
    for key, owner, attr, repl in _optional_targets():
        _originals[key] = getattr(owner, attr)
        setattr(owner, attr, repl)
        _optional_installed.append((key, owner, attr))
    log.info("[foundry] vLLM hooks installed (mode %s)", config.mode.value)


def uninstall_hooks() -> None:
    if not _originals:
        return
    cg, gw, mr = _targets()
    cg.CUDAGraphWrapper.__call__ = _originals.pop("CUDAGraphWrapper.__call__")
    gw.init_worker_distributed_environment = _originals.pop("init_worker_distributed_environment")
    gw.Worker.determine_available_memory = _originals.pop("Worker.determine_available_memory")
    gw.kernel_warmup = _originals.pop("kernel_warmup")
    mr.GPUModelRunner.capture_model = _originals.pop("GPUModelRunner.capture_model")
    mr.GPUModelRunner.load_model = _originals.pop("GPUModelRunner.load_model")
    mr.GPUModelRunner._dummy_run = _originals.pop("GPUModelRunner._dummy_run")
    mr.GPUModelRunner.initialize_kv_cache = _originals.pop("GPUModelRunner.initialize_kv_cache")
    while _optional_installed:
        key, owner, attr = _optional_installed.pop()
        setattr(owner, attr, _originals.pop(key))
    import torch

    torch.cuda.get_device_capability = _originals.pop("torch.cuda.get_device_capability")
    runtime.reset()


def installed() -> bool:
    return bool(_originals)


__all__ = ["install_hooks", "installed", "is_sampler_warmup_run", "nvml_device_capability", "uninstall_hooks"]
