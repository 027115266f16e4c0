"""SGLang integration: persist the CUDA graphs of SGLang's CudaGraphRunner.

``install_hooks(config)`` applies the patches of ``PATCHES`` in this process.
Each names a module, a class (or the module itself) and an attribute; a
patch whose target this SGLang lacks is skipped with a log line unless it is
required. The patches, in the order an SGLang worker reaches them:

  ModelRunner.init_torch_distributed   bind the rank's device, enable the
                                       region (communicator buffers land in
                                       the scratch space), run, skip scratch
  ModelRunnerKVCacheMixin.init_memory_pool
                                       SAVE: record the memory-pool config;
                                       LOAD: apply the recorded one (sizing it
                                       again could move every later address)
  ModelRunner.kernel_warmup            skipped in SAVE and LOAD (its eager
                                       forwards would leave freed segments
                                       LOAD cannot reproduce)
  CudaGraphRunner._create_device_graph SAVE: a foundry graph object
  CudaGraphRunner._capture_graph       SAVE: capture through foundry
  CudaGraphRunner.capture_one_batch_size
                                       SAVE: the two warm-up forwards before
                                       each capture return None instead of
                                       running; the captured graph is saved
                                       under its batch size (and stream index)
  CudaGraphRunner.capture              both: create the DeepEP buffer first
                                       (when DeepEP is the MoE all-to-all);
                                       SAVE: with DeepEP one uncaptured
                                       forward per batch size, then the
                                       FlashInfer per-batch-size metadata
                                       pre-pass and the capture loop reusing
                                       it; manifest + packed modules + final
                                       offset after the loop. LOAD: replaces
                                       the loop: graph pool, preallocate, the
                                       same pre-pass, start all builds,
                                       finish them in SAVE order into
                                       ``graphs`` / ``output_buffers``, set
                                       DeepEP's captured dispatch mode, then
                                       give each graph its own executable on
                                       a background thread (pre-pass and
                                       DeepEP: prepass.py)
  Engine._launch_scheduler_processes,
  DataParallelController.launch_tensor_parallel_group
                                       export LD_PRELOAD (interposer) and the
                                       config path to the spawned schedulers

Parity: reference python/foundry/integration/sglang/hooks.py:67-594 and
config.py:134-142 (workspace rank with and without DP attention). SGLang is
not installed on this build's image: the patches are tested against a fake
SGLang package with the same class and method names
(tests/test_sglang_hooks_cpu.py), not against SGLang itself.
"""

from __future__ import annotations

import dataclasses
import importlib
import logging
import os
import time
from dataclasses import dataclass
from typing import Callable

from ...allocation_region import resume_allocation_region, stop_allocation_region
from .. import graph_ops, runtime
from . import prepass
from ..config import GraphExtensionConfig, GraphExtensionMode

log = logging.getLogger("foundry")

_config: GraphExtensionConfig | None = None
_config_path: str | None = None
_applied: list[tuple[object, str, object]] = []  # (owner, attribute, original)

_CGR = "sglang.srt.model_executor.cuda_graph_runner"
_MR = "sglang.srt.model_executor.model_runner"
_KV = "sglang.srt.model_executor.model_runner_kv_cache_mixin"
_POOL_CFG = "sglang.srt.model_executor.pool_configurator"


def _mode() -> GraphExtensionMode:
    """The rank's mode once its runtime state exists, else the configured one."""
    if runtime.state() is not None:
        return runtime.mode()
    return _config.mode if _config is not None else GraphExtensionMode.NONE


def workspace_rank(server_args, tp_rank: int, pp_rank: int = 0, dp_rank: int | None = None) -> int:
    """Archive folder rank of an SGLang worker. With DP attention the data
    parallel replicas are the attention groups of one TP world, so the rank is
    the worker's place in that world; otherwise replicas stack after each
    other (dp_rank * tp * pp + pp_rank * tp + tp_rank)."""
    tp = int(getattr(server_args, "tp_size", 1) or 1)
    if getattr(server_args, "enable_dp_attention", False):
        return pp_rank * tp + tp_rank
    pp = int(getattr(server_args, "pp_size", 1) or 1)
    return (dp_rank or 0) * tp * pp + pp_rank * tp + tp_rank


def _dp_rank(model_runner) -> int | None:
    r = getattr(model_runner, "dp_rank", None)
    if r is not None:
        return int(r)
    sa = model_runner.server_args
    if not getattr(sa, "enable_dp_attention", False) and int(getattr(sa, "dp_size", 1) or 1) > 1:
        raise RuntimeError("SGLang data parallelism without ModelRunner.dp_rank: the archive rank of this worker "
                           "cannot be derived")
    return None


def suppress_first_calls(fn: Callable, n: int = 2) -> Callable:
    """``fn`` whose first ``n`` calls return None without running it."""
    calls = [0]

    def wrapped(*a, **k):
        calls[0] += 1
        if calls[0] <= n:
            return None
        return fn(*a, **k)

    return wrapped


def sglang_graph_key(bs: int, stream_idx: int | None):
    """The key CudaGraphRunner stores a graph under (batch size, or
    "<stream>_<batch size>" for multi-stream capture)."""
    return bs if stream_idx is None else f"{stream_idx}_{bs}"


# ---- wrappers (original -> replacement) --------------------------------------------------
def _init_torch_distributed(orig):
    def wrapped(self, *a, **k):
        if _mode() == GraphExtensionMode.NONE:
            return orig(self, *a, **k)
        if getattr(self, "device", "cuda") == "cuda" and hasattr(self, "gpu_id"):
            import torch

            torch.cuda.set_device(self.gpu_id)  # the region is reserved on the current device
        rank = workspace_rank(self.server_args, int(self.tp_rank), int(getattr(self, "pp_rank", 0) or 0),
                              _dp_rank(self))
        runtime.setup_graph_extension(_config, rank)
        r = orig(self, *a, **k)
        runtime.skip_to_scratch_boundary()
        return r

    return wrapped


def _memory_pool_config_class(current):
    if current is not None:
        return type(current)
    return importlib.import_module(_POOL_CFG).MemoryPoolConfig


def _init_memory_pool(orig):
    def wrapped(self, *a, **k):
        m = _mode()
        if m == GraphExtensionMode.NONE:
            return orig(self, *a, **k)
        ws = runtime.state().config.workspace_dir
        if m == GraphExtensionMode.LOAD:
            saved = runtime.WarmupState.load(ws)
            cfg = saved.extra.get("memory_pool_config") if saved is not None else None
            if not cfg:
                raise RuntimeError(f"LOAD: {ws} has no recorded memory-pool config (run SAVE first)")
            cls = _memory_pool_config_class(getattr(self, "memory_pool_config", None))
            self.memory_pool_config = cls(**cfg)
            import torch

            torch.cuda.empty_cache()  # SAVE's sizing pass emptied the allocator cache; keep the state alike
            self._apply_memory_pool_config(self.memory_pool_config)
            return None
        r = orig(self, *a, **k)
        state = runtime.WarmupState.load(ws) or runtime.WarmupState()
        state.extra["memory_pool_config"] = dataclasses.asdict(self.memory_pool_config)
        state.save(ws)
        return r

    return wrapped


def _kernel_warmup(orig):
    def wrapped(self, *a, **k):
        if _mode() != GraphExtensionMode.NONE:
            log.info("[foundry] SGLang kernel_warmup skipped (%s)", _mode().value)
            return None
        return orig(self, *a, **k)

    return wrapped


def _create_device_graph(orig):
    def wrapped(self, *a, **k):
        if _mode() == GraphExtensionMode.SAVE:
            from ...graphs import CUDAGraph

            return CUDAGraph()
        return orig(self, *a, **k)

    return wrapped


# True while SAVE's DeepEP warm-up pass runs the capture loop without capturing.
_warmup_pass = [False]


def _capture_graph(orig):
    def wrapped(self, graph, pool, stream, run_once_fn):
        if _warmup_pass[0]:
            return run_once_fn()  # one plain forward: lazy initialisation happens outside any capture
        if _mode() == GraphExtensionMode.SAVE:
            from ...graphs import graph as foundry_graph

            with foundry_graph(graph, pool=pool, stream=stream):
                out = run_once_fn()
            return out
        return orig(self, graph, pool, stream, run_once_fn)

    return wrapped


def _capture_one_batch_size(orig):
    def wrapped(self, bs, forward, stream_idx=None, *a, **k):
        if _mode() != GraphExtensionMode.SAVE:
            return orig(self, bs, forward, stream_idx, *a, **k)
        graph, output = orig(self, bs, suppress_first_calls(forward, 2), stream_idx, *a, **k)
        if _warmup_pass[0]:
            return graph, output
        st = runtime.state()
        key = graph_ops.GraphKey("FULL", int(bs), int(bs), True, False, stream_idx)
        graph.save(os.path.join(st.config.workspace_dir, key.filename(st.capture_index)), output)
        st.capture_index += 1
        return graph, output

    return wrapped


def _load_all_graphs(runner) -> int:
    """LOAD: restores every saved graph of the rank into ``runner.graphs`` /
    ``runner.output_buffers`` in SAVE's capture order."""
    from ...graphs import CUDAGraph

    st = runtime.state()
    plan = graph_ops.start_graph_builds(st.config.workspace_dir)
    by_index = sorted(plan.key_to_index.items(), key=lambda kv: kv[1])
    for key, idx in by_index:
        g, out = CUDAGraph.finish_one_graph_load(plan.pending, idx)
        skey = sglang_graph_key(key.num_tokens, key.piecewise_index)
        runner.graphs[skey] = g
        runner.output_buffers[skey] = out
        st.loaded[key] = (g, out)
    return len(by_index)


def _bind_graph_pool() -> None:
    """LOAD: the graph memory pool SGLang's capture loop would have created
    (its replay and its NCCL allocator look the pool up)."""
    cgr = importlib.import_module(_CGR)
    if not hasattr(cgr, "get_global_graph_memory_pool"):
        return
    if cgr.get_global_graph_memory_pool() is None:
        import torch

        cgr.set_global_graph_memory_pool(torch.cuda.graph_pool_handle())
    try:
        alloc = importlib.import_module("sglang.srt.distributed.device_communicators.pynccl_allocator")
    except ImportError:
        return
    if hasattr(alloc, "set_graph_pool_id"):
        alloc.set_graph_pool_id(cgr.get_global_graph_memory_pool())


def _run_warmup_pass(runner, orig) -> None:
    """SAVE with DeepEP: one plain forward per batch size through SGLang's
    own capture loop, nothing captured or saved, so the lazy initialisation
    SGLang's (suppressed) warm-up forwards would do (DeepGEMM kernels for
    each shape and the like) happens before the real capture. The region is
    paused meanwhile: LOAD runs no such pass, so its activations must not
    move the cursor; the caller empties the allocator cache afterwards."""
    import torch

    saved = runner.graphs, runner.output_buffers
    runner.graphs, runner.output_buffers = {}, {}
    _warmup_pass[0] = True
    t0 = time.perf_counter()
    stop_allocation_region()
    try:
        orig(runner)
        if torch.cuda.is_initialized():
            torch.cuda.synchronize()
    finally:
        resume_allocation_region()
        _warmup_pass[0] = False
        runner.graphs, runner.output_buffers = saved
    log.info("[foundry] SGLang DeepEP warm-up pass: %.3f s", time.perf_counter() - t0)


def _capture(orig):
    def wrapped(self, *a, **k):
        m = _mode()
        if m == GraphExtensionMode.NONE:
            return orig(self, *a, **k)
        import torch

        t0 = time.perf_counter()
        # The same steps, in the same order, up to the capture loop (SAVE) or
        # the graph builds (LOAD), so that what they allocate in the region
        # lands at the same offsets in both runs.
        deepep = prepass.ensure_deepep_buffer(self)
        if m == GraphExtensionMode.LOAD:
            _bind_graph_pool()
            runtime.preallocate_for_load_mode()
        per_bs = prepass.uses_per_batch_metadata(getattr(self, "attn_backend", None))
        restore = None
        if per_bs:
            if m == GraphExtensionMode.SAVE:
                restore = prepass.install_reuse(self)  # pre-pass, then the capture loop reuses it
            else:
                prepass.attention_metadata_prepass(self)
        try:
            if deepep:
                if m == GraphExtensionMode.SAVE:
                    _run_warmup_pass(self, orig)
                torch.cuda.empty_cache()  # drops the warm-up pass's segments; LOAD mirrors the allocator state
            if m == GraphExtensionMode.SAVE:
                r = orig(self, *a, **k)
        finally:
            if restore is not None:
                restore()
        if m == GraphExtensionMode.SAVE:
            graph_ops.finalize_save()
            runtime.capture_final_alloc_offset()
            return r
        n = _load_all_graphs(self)
        if not per_bs and hasattr(self, "attn_backend"):
            # views over the backend's fixed workspace, filled by the loop LOAD replaces
            prepass.attention_metadata_prepass(self)
        adapter = getattr(self, "deepep_adapter", None)
        if adapter is not None:
            adapter.capture(is_extend_in_batch=False)  # the dispatch mode the saved graphs were captured in
        runtime.capture_final_alloc_offset()
        graph_ops.materialize_loaded(background=True)
        log.info("[foundry TIMING] SGLang LOAD of %d graphs: %.3f s", n, time.perf_counter() - t0)
        return None

    return wrapped


def _spawn_site(orig):
    def wrapped(self, *a, **k):
        if _mode() != GraphExtensionMode.NONE:
            os.environ.update(runtime.ld_preload_env(os.environ, _config))
            if _config_path:
                os.environ["FOUNDRY_GRAPH_CONFIG"] = _config_path
                os.environ["FOUNDRY_GRAPH_ENGINE"] = "sglang"
        return orig(self, *a, **k)

    return wrapped


@dataclass(frozen=True)
class Patch:
    module: str
    owner: str  # class name inside the module
    attr: str
    make: Callable
    required: bool = True


PATCHES = [
    Patch(_MR, "ModelRunner", "init_torch_distributed", _init_torch_distributed),
    Patch(_KV, "ModelRunnerKVCacheMixin", "init_memory_pool", _init_memory_pool, required=False),
    Patch(_MR, "ModelRunner", "kernel_warmup", _kernel_warmup, required=False),
    Patch(_CGR, "CudaGraphRunner", "_create_device_graph", _create_device_graph, required=False),
    Patch(_CGR, "CudaGraphRunner", "_capture_graph", _capture_graph, required=False),
    Patch(_CGR, "CudaGraphRunner", "capture_one_batch_size", _capture_one_batch_size),
    Patch(_CGR, "CudaGraphRunner", "capture", _capture),
    Patch("sglang.srt.entrypoints.engine", "Engine", "_launch_scheduler_processes", _spawn_site, required=False),
    Patch("sglang.srt.managers.data_parallel_controller", "DataParallelController",
          "launch_tensor_parallel_group", _spawn_site, required=False),
]


def _resolve(p: Patch):
    try:
        mod = importlib.import_module(p.module)
    except ImportError as e:
        if p.required:
            raise ImportError(f"SGLang module {p.module} is not importable: the SGLang graph extension cannot "
                              "be installed") from e
        return None
    owner = getattr(mod, p.owner, None)
    if owner is None or not hasattr(owner, p.attr):
        if p.required:
            raise ImportError(f"this SGLang has no {p.owner}.{p.attr}: unsupported version")
        return None
    return owner


def install_hooks(config: GraphExtensionConfig | str) -> None:
    """Patches SGLang in this process (idempotent)."""
    global _config, _config_path
    if isinstance(config, (str, os.PathLike)):
        _config_path = os.path.abspath(config)
        config = GraphExtensionConfig.from_toml(config)
    _config = config
    if _applied:
        return
    t0 = os.environ.get("FOUNDRY_SPAWN_T0_NS")
    if t0:
        log.info("[foundry TIMING] process start -> install_hooks: %.1f ms", (time.time_ns() - int(t0)) / 1e6)
    owners = [_resolve(p) for p in PATCHES]  # resolve all first: a missing required target patches nothing
    for p, owner in zip(PATCHES, owners):
        if owner is None:
            log.info("[foundry] SGLang has no %s.%s; patch skipped", p.owner, p.attr)
            continue
        orig = getattr(owner, p.attr)
        _applied.append((owner, p.attr, orig))
        setattr(owner, p.attr, p.make(orig))
    log.info("[foundry] SGLang hooks installed (mode %s, %d patches)", config.mode.value, len(_applied))


def uninstall_hooks() -> None:
    while _applied:
        owner, attr, orig = _applied.pop()
        setattr(owner, attr, orig)
    runtime.reset()


def installed() -> bool:
    return bool(_applied)


__all__ = ["PATCHES", "install_hooks", "installed", "sglang_graph_key", "suppress_first_calls", "uninstall_hooks",
           "workspace_rank"]
