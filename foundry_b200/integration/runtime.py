"""Per-process state of an engine integration: region setup, scratch skip,
warm-up state and the final allocation offset (SAVE writes, LOAD checks).

Order inside an engine worker (both modes):
    setup_graph_extension()      after the device and communicator are up:
                                 LOAD loads the packed modules first, then
                                 both modes enable the region
    skip_to_scratch_boundary()   allocations made so far (communicator
                                 buffers) stay below the scratch boundary
    ... weights, KV cache, graph capture (SAVE) / restore (LOAD) ...
    capture_final_alloc_offset() SAVE: record; LOAD: compare

Parity: reference python/foundry/integration/vllm/runtime.py:48-264.
"""

from __future__ import annotations

import json
import logging
import os
from dataclasses import asdict, dataclass, field

from .. import (get_current_alloc_offset, load_cuda_modules_and_libraries, preallocate_region,
                set_allocation_region, set_current_alloc_offset, set_skip_fatbin_processing)
from ..allocation_region import parse_size
from .config import GraphExtensionConfig, GraphExtensionMode

log = logging.getLogger("foundry")

WARMUP_STATE = "warmup_state.json"
FINAL_OFFSET = "final_alloc_offset.json"


@dataclass
class WarmupState:
    """Engine facts SAVE measured that LOAD must reuse instead of re-measuring
    (re-measuring could change allocation sizes and so every later address)."""

    num_gpu_blocks: int | None = None
    num_cpu_blocks: int | None = None
    extra: dict = field(default_factory=dict)

    def save(self, workspace: str) -> None:
        with open(os.path.join(workspace, WARMUP_STATE), "w") as f:
            json.dump(asdict(self), f, indent=1)

    @classmethod
    def load(cls, workspace: str) -> "WarmupState | None":
        p = os.path.join(workspace, WARMUP_STATE)
        if not os.path.exists(p):
            return None
        with open(p) as f:
            return cls(**json.load(f))


@dataclass
class ExtensionState:
    config: GraphExtensionConfig
    global_rank: int
    capture_index: int = 0
    loaded: dict = field(default_factory=dict)  # strong refs: (graph, output) per key
    pending: object | None = None               # graph_ops.LoadPlan during LOAD


_state: ExtensionState | None = None


def state() -> ExtensionState | None:
    return _state


def mode() -> GraphExtensionMode:
    return _state.config.mode if _state is not None else GraphExtensionMode.NONE


def setup_graph_extension(config: GraphExtensionConfig, global_rank: int) -> ExtensionState:
    global _state
    ws = config.workspace_for(global_rank)
    config.workspace_dir = ws
    if config.mode == GraphExtensionMode.NONE:
        _state = ExtensionState(config, global_rank)
        return _state
    if config.mode == GraphExtensionMode.SAVE:
        os.makedirs(ws, exist_ok=True)
        clear_saved_graphs(ws)
    else:
        if not os.path.isdir(ws):
            raise FileNotFoundError(f"LOAD workspace {ws} does not exist (run SAVE first)")
        set_skip_fatbin_processing(True)
        load_cuda_modules_and_libraries(ws)
    set_allocation_region(config.base_addr, config.region_size)
    _state = ExtensionState(config, global_rank)
    log.info("[foundry] %s rank %d: region %#x + %s, workspace %s", config.mode.value, global_rank,
             config.base_addr, config.region_size, ws)
    return _state


def clear_saved_graphs(workspace: str) -> int:
    """SAVE: removes the graphs, manifest and packed modules of an earlier SAVE
    pass in ``workspace`` (the warm-up state and final offset stay: a second
    pass reuses them to allocate exactly as LOAD will). Returns files removed."""
    n = 0
    for name in os.listdir(workspace):
        if (name.startswith("graph_") and name.endswith((".json", ".cugraph"))) or name in (
                "fatbin_image_packed.img", "fatbin_entrypoint_packed.txt"):
            os.remove(os.path.join(workspace, name))
            n += 1
    return n


def skip_to_scratch_boundary() -> int:
    """Moves the cursor to the scratch boundary (allocations before it - the
    communicator's - may differ between SAVE and LOAD)."""
    cfg = _state.config
    scratch = parse_size(cfg.scratch_space_size)
    cur = get_current_alloc_offset()
    if cur > scratch:
        raise RuntimeError(f"allocations before the scratch boundary ({cur} B) exceed scratch_space_size "
                           f"({scratch} B); raise scratch_space_size")
    set_current_alloc_offset(scratch)
    return scratch


def capture_final_alloc_offset() -> int:
    """SAVE: records the cursor after capture; LOAD: checks it matches."""
    cfg = _state.config
    off = get_current_alloc_offset()
    path = os.path.join(cfg.workspace_dir, FINAL_OFFSET)
    if cfg.mode == GraphExtensionMode.SAVE:
        with open(path, "w") as f:
            json.dump({"final_alloc_offset": off}, f)
    elif cfg.mode == GraphExtensionMode.LOAD and os.path.exists(path):
        with open(path) as f:
            want = json.load(f)["final_alloc_offset"]
        if off != want:
            raise RuntimeError(f"LOAD allocation cursor {off} differs from SAVE {want}: the LOAD run allocated "
                               "differently, restored graphs would point at wrong memory")
    return off


def preallocate_for_load_mode() -> int:
    """LOAD: maps the rest of SAVE's working set in one piece, from the cursor
    to SAVE's final offset, so the weight, KV-cache and graph allocations that
    follow are sub-allocated from it (same addresses, no map call each).
    Returns the bytes mapped (0 outside LOAD or without a recorded offset).

    Parity: reference python/foundry/integration/vllm/runtime.py:235-264."""
    if _state is None or _state.config.mode != GraphExtensionMode.LOAD:
        return 0
    path = os.path.join(_state.config.workspace_dir, FINAL_OFFSET)
    if not os.path.exists(path):
        return 0
    with open(path) as f:
        want = int(json.load(f)["final_alloc_offset"])
    size = want - get_current_alloc_offset()
    if size <= 0:
        return 0
    preallocate_region(size)
    log.info("[foundry] LOAD: preallocated %d MiB up to the SAVE final offset", size >> 20)
    return size


def ld_preload_env(env: dict | None = None, config: GraphExtensionConfig | None = None) -> dict:
    """Environment for a spawned engine process: preload the interposer and
    carry the config path."""
    env = dict(os.environ if env is None else env)
    cfg = config or (_state.config if _state else None)
    lib = cfg.hook_library_path if cfg else None
    if lib:
        pre = env.get("LD_PRELOAD", "")
        if lib not in pre.split(":"):
            env["LD_PRELOAD"] = f"{lib}:{pre}" if pre else lib
    return env


def reset() -> None:
    global _state
    _state = None


__all__ = ["ExtensionState", "WarmupState", "capture_final_alloc_offset", "clear_saved_graphs", "ld_preload_env",
           "mode",
           "preallocate_for_load_mode", "reset", "setup_graph_extension", "skip_to_scratch_boundary", "state"]
