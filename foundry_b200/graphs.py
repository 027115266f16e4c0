"""CUDA graph capture, persistence and restore (Python API).

``CUDAGraph`` captures with torch's graph machinery (so torch's private
memory pools and RNG registration keep working) and hands the captured
``cudaGraph_t`` to the native core, which walks it node by node and can write
it to ``graph_N.json`` + ``graph_N.cugraph``. A later process restores graphs
with ``CUDAGraph.load`` or the two-phase ``start_graph_builds`` /
``finish_graph_loads`` pipeline; restored graphs replay through the native
restore engine (templates + on-demand parameter patches, see csrc/core/restore.h).

Parity: reference python/foundry/graph.py:17-242 (CUDAGraph, graph,
save_graph_manifest) and csrc/binding.cpp:115-338.
"""

from __future__ import annotations

import json
import os
import sys
from typing import Any, Sequence

import torch

from ._native import core

OutputTensors = torch.Tensor | list[torch.Tensor] | tuple[torch.Tensor, ...]

__all__ = ["CUDAGraph", "graph", "save_graph_manifest", "graph_pool_handle"]


def graph_pool_handle():
    return torch.cuda.graph_pool_handle()


def _stream_handle() -> int:
    return torch.cuda.current_stream().cuda_stream


# ---- output tensor metadata --------------------------------------------------------------

def _encode_outputs(outputs: OutputTensors | None) -> str:
    if outputs is None:
        return ""
    if isinstance(outputs, torch.Tensor):
        kind, items = "tensor", [outputs]
    elif isinstance(outputs, (list, tuple)):
        kind, items = ("list" if isinstance(outputs, list) else "tuple"), list(outputs)
    else:
        raise TypeError(f"output_tensors must be a tensor, list or tuple, got {type(outputs)}")
    metas = []
    for t in items:
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise TypeError("output tensors must be CUDA tensors")
        metas.append({
            "data_ptr": t.data_ptr(),
            "sizes": list(t.shape),
            "strides": list(t.stride()),
            "dtype": str(t.dtype).replace("torch.", ""),
            "element_size": t.element_size(),
            "numel": t.numel(),
            "device_type": "cuda",
            "device_index": t.device.index if t.device.index is not None else 0,
            "requires_grad": bool(t.requires_grad),
        })
    return json.dumps({"type": kind, "tensors": metas})


class _DevicePtr:
    """Minimal ``__cuda_array_interface__`` exporter for a raw device byte span."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {
            "data": (ptr, False), "shape": (nbytes,), "typestr": "|u1", "version": 3, "strides": None,
        }


def tensor_from_ptr(ptr: int, sizes: Sequence[int], strides: Sequence[int], dtype: torch.dtype) -> torch.Tensor:
    """Wraps existing device memory as a tensor (no copy, no ownership)."""
    esize = torch.empty((), dtype=dtype).element_size()
    span = 1
    for s, st in zip(sizes, strides):
        if s == 0:
            span = 0
            break
        span += (s - 1) * st
    nbytes = max(span, 1) * esize
    raw = torch.as_tensor(_DevicePtr(ptr, nbytes), device="cuda")
    return raw.view(dtype).as_strided(tuple(sizes), tuple(strides))


def _decode_outputs(text: str) -> OutputTensors | None:
    if not text:
        return None
    meta = json.loads(text)
    tensors = [
        tensor_from_ptr(m["data_ptr"], m["sizes"], m["strides"], getattr(torch, m["dtype"]))
        for m in meta["tensors"]
    ]
    if meta["type"] == "tensor":
        return tensors[0]
    return tensors if meta["type"] == "list" else tuple(tensors)


# ---- random-number generator state ------------------------------------------------------
#
# A captured kernel that draws random numbers reads the Philox seed and offset
# from two device words of its generator's graph state. SAVE records their
# addresses and the graph's whole-graph increment (the offsets one replay
# consumes). LOAD moves those words into a per-device slot owned by this
# module (the restore rewrites the matching pointer words in the kernels'
# parameters), and every replay of a restored graph first writes the
# generator's seed and current offset into the slot and advances the offset,
# which is what torch's own replay does for a captured graph. Restored and
# captured graphs of one process therefore draw the same sequence as the SAVE
# process when the generator starts from the same seed and offset.
# Only the device's default CUDA generator is recorded.

_RNG_SLOTS: dict[int, torch.Tensor] = {}
_RNG_POOLS: dict[int, Any] = {}


def _graph_rng_records(device: int) -> list[dict]:
    """Generator records of the graph whose capture just ended on ``device``."""
    try:
        from . import _torchrng
    except ImportError:  # built by foundry_b200._build; absent only in a partial build
        return []
    st = _torchrng.default_generator_graph_state(device)
    if st["offset_intragraph"] == 0 or not st["seed_ptr"]:
        return []
    return [{"id": 0, "seed": st["seed"], "wholegraph_increment": st["offset_intragraph"],
             "seed_ptr": st["seed_ptr"], "offset_ptr": st["offset_ptr"]}]


def rng_slot(device: int | None = None) -> int:
    """Device address of this process's generator slot (two int64 words) on
    ``device``. Allocated once, from a private pool and outside any active
    allocation region, so it moves neither the region cursor nor the blocks
    of torch's default pool (a LOAD must reproduce SAVE's addresses)."""
    dev = torch.cuda.current_device() if device is None else device
    t = _RNG_SLOTS.get(dev)
    if t is None:
        c = core()
        paused = c.region_active()
        if paused:
            c.stop_allocation_region()
        try:
            pool = torch.cuda.MemPool()
            with torch.cuda.use_mem_pool(pool, device=dev):
                t = torch.zeros(2, dtype=torch.int64, device=dev)
        finally:
            if paused:
                c.resume_allocation_region()
        _RNG_POOLS[dev] = pool
        _RNG_SLOTS[dev] = t
    return t.data_ptr()


def _as_i64(v: int) -> int:
    return v - (1 << 64) if v >= (1 << 63) else v


def _rng_prologue(device: int, increments: list[int]) -> None:
    """Seed/offset words for one replay of a restored graph, then advance."""
    gen = torch.cuda.default_generators[device]
    slot = _RNG_SLOTS[device]
    for inc in increments:
        off = gen.get_offset()
        slot[0].fill_(_as_i64(gen.initial_seed()))
        slot[1].fill_(_as_i64(off))
        gen.set_offset(off + inc)


# ---- CUDAGraph ---------------------------------------------------------------------------

class CUDAGraph:
    """A CUDA graph that can be saved to disk and restored in another process.

    Captured graphs replay through torch; restored graphs through the native
    restore engine. ``save`` requires every kernel of the graph to come from
    an image the module registry saw load (this repository's kernels always
    are; other libraries' kernels are when libfoundry_hook.so is preloaded).
    """

    def __init__(self, keep_graph: bool = False):
        self._keep_graph = keep_graph
        self._torch: torch.cuda.CUDAGraph | None = None
        self._desc = None
        self._analysis_error: str | None = None
        self._restored = None
        self._events_json = ""
        self._rng_device = 0
        self._rng_increments: list[int] = []

    # -- capture ----------------------------------------------------------------------------
    def capture_begin(self, pool=None, capture_error_mode: str = "global") -> None:
        self._torch = torch.cuda.CUDAGraph(keep_graph=True)
        core().start_hook_record()
        self._torch.capture_begin(pool=pool, capture_error_mode=capture_error_mode)

    def capture_end(self) -> None:
        assert self._torch is not None, "capture_begin was not called"
        self._torch.capture_end()
        rng = _graph_rng_records(torch.cuda.current_device())
        c = core()
        c.end_hook_record()
        self._events_json = c.hook_events_json() if c.region_active() else ""
        try:
            self._desc = c.analyze_graph(self._torch.raw_cuda_graph())
            if self._events_json:
                ev = json.loads(self._events_json)
                if ev.get("events"):
                    self._desc.allocator_events_json = self._events_json
            if rng:
                self._desc.generators = rng
        except RuntimeError as e:  # persisted later only if save() is called
            self._desc = None
            self._analysis_error = str(e)
        self._torch.instantiate()

    def register_generator_state(self, generator) -> None:
        if self._torch is None:
            self._torch = torch.cuda.CUDAGraph(keep_graph=True)
        self._torch.register_generator_state(generator)

    def instantiate(self) -> None:
        if self._torch is not None:
            self._torch.instantiate()

    def replay(self) -> None:
        if self._restored is not None:
            if self._rng_increments:
                _rng_prologue(self._rng_device, self._rng_increments)
            self._restored.launch(_stream_handle())
        elif self._torch is not None:
            self._torch.replay()
        else:
            raise RuntimeError("graph was neither captured nor loaded")

    def reset(self) -> None:
        if self._torch is not None:
            self._torch.reset()
        self._torch = None
        self._desc = None
        self._restored = None

    def pool(self):
        if self._torch is None:
            raise RuntimeError("pool() is only available for captured graphs")
        return self._torch.pool()

    def enable_debug_mode(self) -> None:
        if self._torch is not None:
            self._torch.enable_debug_mode()

    def debug_dump(self, debug_path: str) -> None:
        if self._torch is not None:
            self._torch.debug_dump(debug_path)
        elif self._restored is not None:
            with open(debug_path, "w") as f:
                f.write(self._restored.desc.to_json())

    def raw_cuda_graph(self) -> int:
        return self._torch.raw_cuda_graph() if self._torch is not None else 0

    def raw_cuda_graph_exec(self) -> int:
        if self._restored is not None:
            return self._restored.exec_handle
        return self._torch.raw_cuda_graph_exec() if self._torch is not None else 0

    # -- persistence ------------------------------------------------------------------------
    @property
    def desc(self):
        return self._desc if self._restored is None else self._restored.desc

    def save(self, json_path: str, output_tensors: OutputTensors | None = None) -> None:
        """Writes ``json_path`` (JSON) and the ``.cugraph`` binary next to it."""
        if self._desc is None:
            raise RuntimeError(
                f"graph cannot be persisted: {self._analysis_error or 'not captured'}"
            )
        self._desc.output_tensors_json = _encode_outputs(output_tensors)
        os.makedirs(os.path.dirname(os.path.abspath(json_path)), exist_ok=True)
        self._desc.save(json_path)

    @classmethod
    def _from_restored(cls, restored) -> tuple["CUDAGraph", OutputTensors | None]:
        g = cls()
        g._restored = restored
        g._rng_device = torch.cuda.current_device()
        g._rng_increments = [r["wholegraph_increment"] for r in restored.desc.generators if r["seed_ptr"]]
        return g, _decode_outputs(restored.output_tensors_json)

    @staticmethod
    def load(json_path: str, pool=None) -> "CUDAGraph | tuple[CUDAGraph, OutputTensors]":
        torch.cuda.synchronize()
        restored = core().load_graph(json_path, rng_slot())
        g, outputs = CUDAGraph._from_restored(restored)
        return g if outputs is None else (g, outputs)

    @staticmethod
    def start_graph_builds(json_paths: list[str], pool=None, num_threads: int = 4):
        """Reads every graph (in parallel) and starts building templates on a
        background thread; returns immediately with a pending handle."""
        torch.cuda.synchronize()
        return core().start_graph_builds(list(json_paths), num_threads, rng_slot())

    @staticmethod
    def finish_one_graph_load(pending, index: int) -> tuple["CUDAGraph", OutputTensors | None]:
        """Finishes graph ``index``: waits for the builds, replays its allocator
        events (call in SAVE capture order), rebuilds its output tensors."""
        return CUDAGraph._from_restored(pending.finish_one(index))

    @staticmethod
    def finish_graph_loads(pending) -> list[tuple["CUDAGraph", OutputTensors | None]]:
        return [CUDAGraph.finish_one_graph_load(pending, i) for i in range(pending.num_graphs)]

    def materialize(self) -> None:
        """Gives a restored graph its own executable (no parameter patching on
        later replays). Safe to call from a background thread."""
        if self._restored is not None:
            self._restored.materialize()


class graph:
    """Context manager capturing into a ``CUDAGraph`` on a side stream."""

    default_capture_stream: torch.cuda.Stream | None = None

    def __init__(self, cuda_graph: CUDAGraph, pool=None, stream: torch.cuda.Stream | None = None,
                 capture_error_mode: str = "global"):
        if self.__class__.default_capture_stream is None:
            self.__class__.default_capture_stream = torch.cuda.Stream()
        self.pool = () if pool is None else (pool,)
        self.capture_stream = stream if stream is not None else self.__class__.default_capture_stream
        self.stream_ctx = torch.cuda.stream(self.capture_stream)
        self.cuda_graph = cuda_graph
        self.capture_error_mode = capture_error_mode

    def __enter__(self) -> None:
        # No empty_cache here: the region cursor only moves forward, so freeing
        # between captures would inflate the final offset without reusing memory.
        torch.cuda.synchronize()
        self.stream_ctx.__enter__()
        self.cuda_graph.capture_begin(*self.pool, capture_error_mode=self.capture_error_mode)

    def __exit__(self, *args) -> None:
        self.cuda_graph.capture_end()
        self.stream_ctx.__exit__(*args)


def _graph_index(name: str) -> int:
    try:
        return int(name.split("_")[1].split(".")[0])
    except (IndexError, ValueError):
        return 1 << 30


def _manifest_candidates(archive_dir: str) -> list[str]:
    names = [f for f in os.listdir(archive_dir)
             if f.startswith("graph_") and f.endswith(".json") and f != "graph_manifest.json"]
    return sorted(names, key=lambda f: (_graph_index(f), f))


def save_graph_manifest(archive_dir: str) -> dict[str, Any] | None:
    """Writes ``graph_manifest.json`` for the graphs saved in ``archive_dir``.

    Graphs with equal topology keys form one group; the lowest-numbered graph
    of a group is its template (restored as a real executable) and the others
    are restored as parameter patches onto it. A member's JSON no longer
    needs its dependency table, so it is dropped there (the ``.cugraph``
    binary keeps it). Returns the manifest, or None when the folder holds no
    graph. Raises ``ValueError`` when a graph has no topology key: such an
    archive could only be restored one graph at a time, and a manifest that
    silently left graphs out would hide that.

    Manifest schema (kept from reference python/foundry/graph.py:170-242 so
    either side reads the other's archives):
    ``{"topology_groups": [{"topology_key", "template", "members"}]}``.
    """
    names = _manifest_candidates(archive_dir)
    if not names:
        return None
    docs = {}
    for name in names:
        with open(os.path.join(archive_dir, name)) as f:
            docs[name] = json.load(f)
    keyless = [n for n in names if not docs[n].get("topology_key")]
    if keyless:
        raise ValueError(f"{archive_dir}: {len(keyless)} graph(s) have no topology_key "
                         f"(first: {keyless[0]}); re-save them with this version")
    order: list[str] = []
    members: dict[str, list[str]] = {}
    for name in names:
        key = docs[name]["topology_key"]
        if key not in members:
            order.append(key)
            members[key] = []
        members[key].append(name)
    manifest = {"topology_groups": [{"topology_key": k, "template": members[k][0], "members": members[k]}
                                    for k in order]}
    dropped = 0
    for group in manifest["topology_groups"]:
        for name in group["members"][1:]:
            if docs[name].pop("dependencies", None) is None:
                continue
            _write_json_atomic(os.path.join(archive_dir, name), docs[name], indent=None)
            dropped += 1
    _write_json_atomic(os.path.join(archive_dir, "graph_manifest.json"), manifest, indent=2)
    patched = len(names) - len(order)
    print(f"[foundry_b200] manifest: {len(names)} graphs, {len(order)} topology groups, "
          f"{patched} restored by patching a template; edge lists dropped from {dropped} member JSON files",
          file=sys.stderr)
    return manifest


def _write_json_atomic(path: str, obj: Any, indent: int | None) -> None:
    tmp = f"{path}.tmp.{os.getpid()}"
    with open(tmp, "w") as f:
        json.dump(obj, f, indent=indent)
    os.replace(tmp, path)
