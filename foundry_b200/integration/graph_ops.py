"""Engine-agnostic graph operations of the integrations: the archive file
naming of captured graphs, capture-or-load of one graph, the LOAD pipeline
(start all builds, finish each graph when the engine asks for it) and the
SAVE finalisation (manifest + packed modules).

File names encode everything LOAD needs to match a captured graph to the
engine's request (mode, tokens, requests, uniform decode, LoRA, piecewise
index), the same scheme as the reference
(python/foundry/integration/vllm/graph_ops.py:76-115):

    graph_<i>_<MODE>_t<tokens>_r<reqs|N>_<U|X><L|X>_pc<index|N>.json
"""

from __future__ import annotations

import os
import re
from dataclasses import dataclass
from typing import Any, Callable

import torch

from .. import pack_fatbins_to_folder
from ..graphs import CUDAGraph, graph as foundry_graph, save_graph_manifest
from . import runtime
from .config import GraphExtensionMode


@dataclass(frozen=True)
class GraphKey:
    """Identity of one captured graph inside an engine."""

    mode: str                 # engine's runtime mode name, e.g. FULL / PIECEWISE
    num_tokens: int
    num_reqs: int | None = None
    uniform: bool = False
    has_lora: bool = False
    piecewise_index: int | None = None

    def filename(self, index: int) -> str:
        r = "N" if self.num_reqs is None else str(self.num_reqs)
        pc = "N" if self.piecewise_index is None else str(self.piecewise_index)
        return (f"graph_{index}_{self.mode}_t{self.num_tokens}_r{r}_{'U' if self.uniform else 'X'}"
                f"{'L' if self.has_lora else 'X'}_pc{pc}.json")


_NAME = re.compile(r"^graph_(\d+)_([A-Z_]+)_t(\d+)_r(\d+|N)_([UX])([LX])_pc(\d+|N)\.json$")


def parse_filename(name: str) -> tuple[int, GraphKey] | None:
    m = _NAME.match(os.path.basename(name))
    if not m:
        return None
    idx, mode, tok, req, u, lora, pc = m.groups()
    return int(idx), GraphKey(mode, int(tok), None if req == "N" else int(req), u == "U", lora == "L",
                              None if pc == "N" else int(pc))


@dataclass
class LoadPlan:
    pending: Any
    key_to_index: dict
    paths: list


def start_graph_builds(workspace: str, num_threads: int = 8) -> LoadPlan:
    """LOAD: parallel read of every graph file of the workspace and background
    template builds; graphs are finished one by one by ``capture_or_load``.
    A second call in the same process returns the plan already started."""
    st = runtime.state()
    if st is not None and st.pending is not None:
        return st.pending
    found = []
    for name in os.listdir(workspace):
        p = parse_filename(name)
        if p is not None:
            found.append((p[0], p[1], os.path.join(workspace, name)))
    found.sort(key=lambda x: x[0])
    paths = [f[2] for f in found]
    pending = CUDAGraph.start_graph_builds(paths, num_threads=num_threads) if paths else None
    plan = LoadPlan(pending, {f[1]: i for i, f in enumerate(found)}, paths)
    if st is not None:
        st.pending = plan
    return plan


def capture_or_load(key: GraphKey, runnable: Callable, args: tuple = (), kwargs: dict | None = None, pool=None,
                    stream=None):
    """Returns (graph, output) for ``key``: a plain torch graph (mode none), a
    captured-and-saved foundry graph (save) or the restored graph (load)."""
    kwargs = kwargs or {}
    mode = runtime.mode()
    if mode == GraphExtensionMode.NONE:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=pool, stream=stream):
            out = runnable(*args, **kwargs)
        return g, out
    st = runtime.state()
    if mode == GraphExtensionMode.SAVE:
        g = CUDAGraph()
        with foundry_graph(g, pool=pool, stream=stream):
            out = runnable(*args, **kwargs)
        g.save(os.path.join(st.config.workspace_dir, key.filename(st.capture_index)), out)
        st.capture_index += 1
        return g, out
    plan = st.pending
    if plan is None:
        raise RuntimeError("LOAD: start_graph_builds() was not called before the first graph request")
    idx = plan.key_to_index.get(key)
    if idx is None:
        raise KeyError(f"LOAD: no saved graph for {key}; saved: {sorted(plan.key_to_index, key=str)[:8]} ...")
    g, out = CUDAGraph.finish_one_graph_load(plan.pending, idx)
    st.loaded[key] = (g, out)  # keep region-backed outputs alive for the engine's weak references
    return g, out


def materialize_loaded(background: bool = True):
    """LOAD: gives every graph restored so far its own executable (largest
    token count first), so the engine's later batch-size switches patch
    nothing. With ``background`` on a daemon thread, which is returned;
    launches may run concurrently."""
    import threading

    st = runtime.state()
    if st is None or not st.loaded:
        return None
    graphs = [g for _, (g, _) in sorted(st.loaded.items(), key=lambda kv: -kv[0].num_tokens)]

    def run():
        for g in graphs:
            if hasattr(g, "materialize"):
                g.materialize()

    if not background:
        run()
        return None
    t = threading.Thread(target=run, name="foundry-materialize", daemon=True)
    t.start()
    return t


def finalize_save(workspace: str | None = None) -> None:
    """SAVE: graph manifest (topology groups) + packed modules of the workspace."""
    st = runtime.state()
    ws = workspace or st.config.workspace_dir
    save_graph_manifest(ws)
    pack_fatbins_to_folder(ws)


__all__ = ["GraphKey", "LoadPlan", "capture_or_load", "finalize_save", "materialize_loaded", "parse_filename",
           "start_graph_builds"]
