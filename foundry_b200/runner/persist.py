"""SAVE / LOAD of a serving engine's decode graphs.

Archive layout (one directory per rank, like the reference's workspace
``rank_N``): ``graph_<i>.json`` + ``graph_<i>.cugraph`` for the i-th decode
batch size, ``graph_manifest.json``, ``fatbin_image_packed.img``,
``fatbin_entrypoint_packed.txt`` and ``runner_state.json`` (engine config,
arena layout and final region offset - the role of the reference's
warmup_state.json and final_alloc_offset.json,
python/foundry/integration/vllm/runtime.py:48-99, 214-227).

LOAD overlaps the work that does not depend on each other: image loading and
region setup first (they fix every address), then the graph restore runs on
the native background thread while weights are (re)initialised on the GPU.
"""

from __future__ import annotations

import json
import os
import time

import torch

from .. import core, load_cuda_modules_and_libraries, pack_fatbins_to_folder
from ..graphs import CUDAGraph, save_graph_manifest
from ..utils.trace import phase
from ..models import config_from_dict
from .engine import EngineConfig, LLMEngine

STATE_FILE = "runner_state.json"


def engine_config_to_dict(e: EngineConfig) -> dict:
    return {
        "model": e.model.to_dict(), "max_batch": e.max_batch, "max_seq_len": e.max_seq_len,
        "num_blocks": e.num_blocks, "max_prefill_tokens": e.max_prefill_tokens,
        "max_prefill_seqs": e.max_prefill_seqs, "graph_sizes": e.graph_sizes, "region_base": e.region_base,
        "region_size": e.region_size, "seed": e.seed, "tp": e.tp, "ep": e.ep,
    }


def engine_config_from_dict(d: dict) -> EngineConfig:
    d = dict(d)
    d["model"] = config_from_dict(d["model"])
    return EngineConfig(**d)


def _layout_fingerprint(eng: LLMEngine) -> dict:
    return {
        "embed_ptr": eng.weights.embed.data_ptr(),
        "state_ptr": eng.state.input_ids.data_ptr(),
        "k_cache0_ptr": eng.k_cache[0].data_ptr(),
        "arena_used": eng.arena.used,
        "final_alloc_offset": core().get_current_alloc_offset(),
        "symm": (eng.tp or eng.ep).symm.layout() if (eng.tp or eng.ep) is not None else None,
    }


def rank_dir(archive: str) -> str:
    """Per-rank subfolder of a tensor-parallel archive (``rank_<r>``); the
    archive itself for a single-rank engine."""
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        sub = os.path.join(archive, f"rank_{dist.get_rank()}")
        if os.path.isdir(sub) or not os.path.exists(os.path.join(archive, STATE_FILE)):
            return sub
    return archive


def save(eng: LLMEngine, archive: str) -> dict:
    """Captures (if needed) and writes every decode graph of ``eng``; a
    tensor-parallel engine writes its rank's graphs under ``rank_<r>``."""
    if eng.ecfg.tp > 1 or eng.ecfg.ep > 1:
        archive = os.path.join(archive, f"rank_{(eng.tp or eng.ep).rank}")
    os.makedirs(archive, exist_ok=True)
    t0 = time.perf_counter()
    capture_s = 0.0
    if not eng.graphs:
        with phase("foundry.save.capture"):
            capture_s = eng.capture_graphs()
    t1 = time.perf_counter()
    paths = []
    for i, s in enumerate(eng.graph_sizes):
        p = os.path.join(archive, f"graph_{i}.json")
        eng.graphs[s].save(p, output_tensors=eng.state.next_ids[:s])
        paths.append(p)
    pack_fatbins_to_folder(archive)
    save_graph_manifest(archive)
    state = {
        "engine": engine_config_to_dict(eng.ecfg),
        "graph_sizes": eng.graph_sizes,
        "layout": _layout_fingerprint(eng),
        "capture_s": capture_s,
        "save_s": time.perf_counter() - t1,
    }
    with open(os.path.join(archive, STATE_FILE), "w") as f:
        json.dump(state, f, indent=1)
    state["total_s"] = time.perf_counter() - t0
    return state


def load(archive: str, init_weights: bool = True, num_threads: int = 8) -> tuple[LLMEngine, dict]:
    """Rebuilds the engine at the SAVE addresses and restores its decode graphs."""
    t0 = time.perf_counter()
    archive = rank_dir(archive)
    with open(os.path.join(archive, STATE_FILE)) as f:
        state = json.load(f)
    ecfg = engine_config_from_dict(state["engine"])
    torch.cuda.init()
    with phase("foundry.load.modules"):
        load_cuda_modules_and_libraries(archive)
    t_mod = time.perf_counter()
    with phase("foundry.load.engine_layout"):
        eng = LLMEngine(ecfg, init_weights=False)
    lay = _layout_fingerprint(eng)
    for k in ("embed_ptr", "state_ptr", "k_cache0_ptr", "arena_used"):
        if lay[k] != state["layout"][k]:
            raise RuntimeError(f"LOAD layout differs from SAVE at {k}: {lay[k]:#x} vs {state['layout'][k]:#x}")
    if lay["symm"] != state["layout"].get("symm"):
        raise RuntimeError(f"symmetric-memory layout differs from SAVE: {lay['symm']} vs {state['layout'].get('symm')}")
    t_arena = time.perf_counter()
    paths = [os.path.join(archive, f"graph_{i}.json") for i in range(len(state["graph_sizes"]))]
    with phase("foundry.load.start_graph_builds"):
        pending = CUDAGraph.start_graph_builds(paths, num_threads=num_threads)
    if init_weights:
        with phase("foundry.load.init_weights"):
            eng.init_weights()  # GPU work overlaps the background template builds
    with phase("foundry.load.finish_graph_loads"):
        loaded = CUDAGraph.finish_graph_loads(pending)
    for s, (g, _) in zip(state["graph_sizes"], loaded):
        eng.graphs[s] = g
    eng.materialize_after_first_step = True
    t_done = time.perf_counter()
    timings = {
        "modules_s": t_mod - t0,
        "arena_s": t_arena - t_mod,
        "restore_s": t_done - t_arena,
        "restore_phase1_ms": pending.phase1_ms,
        "restore_phase2_ms": pending.phase2_ms,
        "num_graphs": len(paths),
        "num_groups": pending.num_groups,
        "load_total_s": t_done - t0,
    }
    return eng, timings
