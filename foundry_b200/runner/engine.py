"""Serving engine: static arena, paged KV cache, prefill + graph-replayed decode.

Design (B200-first):
  * one process per GPU; all device memory comes from a static arena in the
    deterministic VMM region, so decode graphs captured in one process
    replay in another after a restore;
  * KV cache pages of 64 tokens, laid out [blocks, kv_heads, 64, 128] per
    layer so one (block, head) page is a contiguous 16 KB burst;
  * pages for a request (prompt + max_new_tokens) are reserved at admission,
    so a decode step needs no host-side table updates;
  * a decode step is one CUDA-graph launch: position/slot bookkeeping,
    32 layers, lm_head and argmax all run inside the graph; the host only
    copies in the step's input tokens and reads back the sampled ones.

Parity: the reference has no runner (it patches vLLM/SGLang); this plays the
role of the engine whose decode graphs it persists (reference
python/foundry/integration/vllm/graph_ops.py:123-205 capture-or-load loop).
"""

from __future__ import annotations

import math
import threading
import time
from dataclasses import dataclass, field

import torch

from .. import ops
from ..models import family
from ..models.llama import LlamaConfig, LlamaWeights
from ..ops.attention import PREFILL_TILE, DecodeWorkspace, decode_splits, prefill_tiles
from ..ops.gemm import MAX_SPLITS, SWIGLU_SK_ENABLED, PartialBuffer, swiglu_sk_sizes
from .arena import Arena

PAGE = 64
# prefill attention kernel: "tc" (tcgen05) or "simt" (CUDA cores)
PREFILL_IMPL = __import__("os").environ.get("FOUNDRY_PREFILL_ATTN", "tc")
EP_PREFILL_CAP = 2048  # prefill tokens per chunk and rank under expert parallelism (sizes the exchange)


def default_graph_sizes(max_batch: int = 1024) -> list[int]:
    """{1, 2, 4, 8} + 16..max_batch step 16: 67 sizes for 1024."""
    sizes = [s for s in (1, 2, 4, 8) if s <= max_batch]
    sizes += list(range(16, max_batch + 1, 16))
    return sizes


@dataclass
class EngineConfig:
    model: LlamaConfig
    max_batch: int = 256            # largest decode batch (graph sizes are capped by it)
    max_seq_len: int = 640          # prompt + generated tokens per request
    num_blocks: int | None = None   # KV pages; default: max_batch * pages per seq
    max_prefill_tokens: int = 8192
    max_prefill_seqs: int = 64
    graph_sizes: list[int] | None = None
    region_base: int | None = 0x600000000000
    region_size: int | str = "96GB"
    seed: int = 0
    tp: int = 1                     # tensor-parallel ranks (= torch.distributed world)
    ep: int = 1                     # expert-parallel ranks (MoE; attention is data-parallel)
    extra: dict = field(default_factory=dict)

    @property
    def pages_per_seq(self) -> int:
        return math.ceil(self.max_seq_len / PAGE)


def _model_buffers(obj, cfg, w, arena, rows) -> None:
    """Allocates the model family's extra scratch and, under expert
    parallelism, the exchange's per-state scratch (zeroed: padding rows of a
    GEMM tile are read, never NaN bit patterns)."""
    spec = getattr(family(cfg)[2], "buffers", None)
    items = dict(spec(cfg, w, rows)) if spec is not None else {}
    ep = getattr(obj, "ep", None)
    if ep is not None:
        items.update(ep.buffers(rows))
    for name, (shape, dtype) in items.items():
        setattr(obj, name, arena.zeros(shape, dtype))
    if ep is not None:
        obj.ep_ident.copy_(torch.arange(obj.ep_ident.numel(), dtype=torch.int32))


class TPContext:
    """Exchange buffers of a tensor-parallel engine in symmetric memory:
    barrier control words, the (value, index) pairs of the sharded argmax and
    the two alternating slot buffers of the row-parallel GEMMs (o, down)."""

    def __init__(self, rows: int, hidden: int, pair_rows: int, group=None):
        from ..parallel.comm import SlotExchange
        from ..parallel.symm import CTRL_BYTES, SymmetricMemory
        import torch.distributed as dist

        from ..parallel.comm import AR_BLOCK_BYTES

        world = dist.get_world_size(group)
        pairs_bytes = -(-(world * pair_rows * 8) // 4096) * 4096
        slot_off = CTRL_BYTES + pairs_bytes
        ar_off = -(-(slot_off + 2 * world * rows * hidden * 2) // 4096) * 4096
        self.symm = SymmetricMemory(ar_off + 2 * AR_BLOCK_BYTES, group)
        self.pairs_offset = CTRL_BYTES
        self.slots = SlotExchange(self.symm, slot_off, rows, hidden, ar_offset=ar_off)
        self.rank, self.world = self.symm.rank, world
        # counters of the fused GEMM + all-reduce start at zero on every rank
        if self.symm.mock:
            import ctypes

            ctypes.memset(self.symm.ptr(self.rank, ar_off), 0, 2 * AR_BLOCK_BYTES)
        else:
            self.symm.tensor(self.rank, (2 * AR_BLOCK_BYTES,), torch.uint8, ar_off).zero_()
            torch.cuda.synchronize()
        dist.barrier(group=group)

    def close(self) -> None:
        self.symm.close()


class DecodeState:
    """Static device buffers of a decode step for up to max_batch rows
    (per-rank shapes under tensor parallelism)."""

    def __init__(self, ecfg: EngineConfig, arena: Arena, k_cache, v_cache, w: LlamaWeights, tp=None, ep=None):
        cfg = ecfg.model
        b = ecfg.max_batch
        self.tp = tp
        self.ep = ep
        nq, nkv = w.nq_l, w.nkv_l
        self.page = PAGE
        self.max_pages = ecfg.pages_per_seq
        i32 = torch.int32
        self.input_ids = arena.zeros((b,), i32)
        self.next_ids = arena.zeros((b,), i32)
        self.seq_lens = arena.zeros((b,), i32)
        self.positions = arena.zeros((b,), i32)
        self.slots = arena.zeros((b,), i32)
        self.active = arena.zeros((b,), i32)
        self.block_tables = arena.zeros((b, self.max_pages), i32)
        self.hidden = arena.empty((b, cfg.hidden))
        self.normed = arena.empty((b, cfg.hidden))
        self.qkv = arena.empty((b, w.qkv_dim_l))
        self.q = arena.empty((b, nq, cfg.head_dim))
        self.attn_out = arena.empty((b, nq * cfg.head_dim))
        if w.inter_l:
            self.gate_up = arena.empty((b, 2 * w.inter_l))
            self.act = arena.empty((b, w.inter_l))
        self.logits = arena.empty((b, w.vocab_l))
        self.k_cache, self.v_cache = k_cache, v_cache
        _model_buffers(self, ecfg.model, w, arena, b)
        # fp32 split-K slices of the decode GEMMs (consumed by the next op)
        part_n = MAX_SPLITS * b * max(w.qkv_dim_l, cfg.hidden)
        sk_ws_n, sk_fl_n = swiglu_sk_sizes(w.inter_l) if w.inter_l and SWIGLU_SK_ENABLED else (0, 0)
        self.part = PartialBuffer(buf=arena.empty((max(part_n, sk_ws_n),), torch.float32))
        # stream-K GEMMs (gate_up, lm_head, and the fused gate/up + SwiGLU
        # when FOUNDRY_SWIGLU_SK=1) keep their partial tiles in the split-K
        # slice buffer (free between the ops that use it) and their tickets in
        # zeroed flag arrays that every launch leaves zeroed
        self.sk = ops.StreamKBuffer(self.part.buf, arena.zeros((1024 * 8,), torch.int32))
        self.swiglu_sk = (ops.StreamKBuffer(self.part.buf, arena.zeros((sk_fl_n,), torch.int32))
                          if sk_fl_n else None)
        sizes = ecfg.graph_sizes or default_graph_sizes(b)
        self.attn_splits = {s: decode_splits(s, nkv, self.max_pages) for s in sizes}
        for s in range(1, b + 1):
            self.attn_splits.setdefault(s, decode_splits(s, nkv, self.max_pages))
        cap = max(s * nq * sp for s, (sp, _) in self.attn_splits.items())
        self.attn_ws = DecodeWorkspace(
            b, nq, 1, o_part=arena.empty((cap * 128,), torch.float32),
            ml_part=arena.empty((cap * 2,), torch.float32))
        self.attn_ws.capacity = cap


class PrefillBatch:
    """Static device buffers of one packed prefill chunk."""

    def __init__(self, ecfg: EngineConfig, arena: Arena, k_cache, v_cache, w: LlamaWeights, tp=None, ep=None):
        cfg = ecfg.model
        t, n = ecfg.max_prefill_tokens, ecfg.max_prefill_seqs
        self.tp = tp
        self.ep = ep
        nq, nkv = w.nq_l, w.nkv_l
        i32 = torch.int32
        self.max_tokens, self.max_seqs = t, n
        self.input_ids = arena.zeros((t,), i32)
        self.positions = arena.zeros((t,), i32)
        self.slots = arena.zeros((t,), i32)
        self.cu_seqlens = arena.zeros((n + 1,), i32)
        max_tiles = t // 64 + n
        self.tile_seq = arena.zeros((max_tiles,), i32)
        self.tile_start = arena.zeros((max_tiles,), i32)
        self.last_rows = arena.zeros((n,), torch.int64)
        self.hidden = arena.empty((t, cfg.hidden))
        self.normed = arena.empty((t, cfg.hidden))
        self.qkv = arena.empty((t, w.qkv_dim_l))
        self.q = arena.empty((t, nq, cfg.head_dim))
        self.k_rot = arena.empty((t, nkv, cfg.head_dim))
        self.v_rot = arena.empty((t, nkv, cfg.head_dim))
        self.attn_out = arena.empty((t, nq * cfg.head_dim))
        if w.inter_l:
            self.gate_up = arena.empty((t, 2 * w.inter_l))
            self.act = arena.empty((t, w.inter_l))
        _model_buffers(self, cfg, w, arena, t)
        self.last_hidden = arena.empty((n, cfg.hidden))
        self.last_normed = arena.empty((n, cfg.hidden))
        self.logits = arena.empty((n, w.vocab_l))
        self.next_ids = arena.zeros((n,), i32)
        self.k_cache, self.v_cache = k_cache, v_cache
        self.num_tokens = 0
        self.num_seqs = 0
        # host staging (pinned)
        self.h_ids = torch.zeros(t, dtype=i32, pin_memory=True)
        self.h_pos = torch.zeros(t, dtype=i32, pin_memory=True)
        self.h_slots = torch.zeros(t, dtype=i32, pin_memory=True)
        self.h_cu = torch.zeros(n + 1, dtype=i32, pin_memory=True)
        self.h_tile_seq = torch.zeros(max_tiles, dtype=i32, pin_memory=True)
        self.h_tile_start = torch.zeros(max_tiles, dtype=i32, pin_memory=True)
        self.h_last = torch.zeros(n, dtype=torch.int64, pin_memory=True)
        self.h_next = torch.zeros(n, dtype=i32, pin_memory=True)


@dataclass
class Request:
    rid: int
    prompt: list[int]
    max_new_tokens: int
    output: list[int] = field(default_factory=list)
    row: int = -1            # decode row
    pages: list[int] = field(default_factory=list)

    @property
    def done(self) -> bool:
        return len(self.output) >= self.max_new_tokens


class LLMEngine:
    def __init__(self, ecfg: EngineConfig, init_weights: bool = True):
        self.ecfg = ecfg
        cfg = ecfg.model
        torch.cuda.init()
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.arena = Arena(ecfg.region_base, ecfg.region_size, self.device)
        t0 = time.perf_counter()
        self.tp = None
        tp_rank = 0
        if ecfg.tp > 1:
            import torch.distributed as dist

            if not dist.is_initialized() or dist.get_world_size() != ecfg.tp:
                raise RuntimeError(f"tp={ecfg.tp} needs an initialised process group of that size")
            tp_rank = dist.get_rank()
            # Symmetric buffers live at fixed addresses outside the arena.
            self.tp = TPContext(max(ecfg.max_batch, ecfg.max_prefill_tokens), cfg.hidden,
                                max(ecfg.max_batch, ecfg.max_prefill_seqs))
        # Order matters: it fixes every device address (SAVE == LOAD).
        _, weights_cls, model_cls = family(cfg)
        kw = {}
        self.ep = None
        if ecfg.ep > 1:
            import torch.distributed as dist

            from ..parallel.ep import EPContext

            if ecfg.tp > 1 or not dist.is_initialized() or dist.get_world_size() != ecfg.ep:
                raise RuntimeError(f"ep={ecfg.ep} needs tp=1 and an initialised process group of that size")
            kw = {"ep_rank": dist.get_rank(), "ep_size": ecfg.ep}
            ecfg.max_prefill_tokens = min(ecfg.max_prefill_tokens, EP_PREFILL_CAP)
            self.ep = EPContext(cfg, max(ecfg.max_batch, ecfg.max_prefill_tokens))
        self.weights = weights_cls(cfg, self.arena, seed=ecfg.seed, init=init_weights, tp_rank=tp_rank,
                                   tp_size=ecfg.tp, **kw)
        nb = ecfg.num_blocks or ecfg.max_batch * ecfg.pages_per_seq
        self.num_blocks = nb
        nkv = self.weights.nkv_l
        # Zeroed once: cache slots past a sequence's end are read (and masked) by
        # the attention kernels, so they must never hold NaN bit patterns.
        self.k_cache = [self.arena.zeros((nb, nkv, PAGE, cfg.head_dim)) for _ in range(cfg.layers)]
        self.v_cache = [self.arena.zeros((nb, nkv, PAGE, cfg.head_dim)) for _ in range(cfg.layers)]
        self.cos_sin = self.arena.empty((ecfg.max_seq_len, cfg.head_dim // 2, 2), torch.float32)
        self.cos_sin.copy_(ops.rope_cos_sin(ecfg.max_seq_len, cfg.rope_theta, cfg.head_dim,
                                            scaling=cfg.rope_scaling))
        self.state = DecodeState(ecfg, self.arena, self.k_cache, self.v_cache, self.weights, self.tp, self.ep)
        self.prefill_buf = PrefillBatch(ecfg, self.arena, self.k_cache, self.v_cache, self.weights, self.tp, self.ep)
        self.model = model_cls(cfg, self.weights, self.cos_sin)
        self.graph_sizes = sorted(ecfg.graph_sizes or default_graph_sizes(ecfg.max_batch))
        self.graphs: dict[int, object] = {}
        # Restored graphs share one executable per topology group and patch
        # their differing nodes in when the batch size changes. After the
        # first decode step a background thread gives every graph its own
        # executable (largest batch first), so later switches cost nothing.
        self.materialize_after_first_step = False
        self._materializer: threading.Thread | None = None
        self._stop_materializing = False
        # Under expert parallelism page 0 is kept for the padding prefill
        # chunks that keep every rank's collective steps in step.
        self.free_pages = list(range(nb - 1, 0 if self.ep is not None else -1, -1))
        self.rows_free = list(range(ecfg.max_batch - 1, -1, -1))
        self.running: list[Request] = []
        self.h_in = torch.zeros(ecfg.max_batch, dtype=torch.int32, pin_memory=True)
        self.h_out = torch.zeros(ecfg.max_batch, dtype=torch.int32, pin_memory=True)
        self.h_tables = torch.zeros(ecfg.max_batch, ecfg.pages_per_seq, dtype=torch.int32, pin_memory=True)
        self.h_lens = torch.zeros(ecfg.max_batch, dtype=torch.int32, pin_memory=True)
        self.h_active = torch.zeros(ecfg.max_batch, dtype=torch.int32, pin_memory=True)
        self.setup_s = time.perf_counter() - t0

    def init_weights(self) -> None:
        self.weights.init(self.ecfg.seed)

    # ---- requests ------------------------------------------------------------------------------
    def add_requests(self, prompts: list[list[int]], max_new_tokens: int) -> list[Request]:
        reqs = []
        for p in prompts:
            if len(p) + max_new_tokens > self.ecfg.max_seq_len:
                raise ValueError("request longer than max_seq_len")
            n_pages = math.ceil((len(p) + max_new_tokens) / PAGE)
            if n_pages > len(self.free_pages) or not self.rows_free:
                raise RuntimeError("out of KV pages or decode rows")
            r = Request(rid=len(reqs), prompt=list(p), max_new_tokens=max_new_tokens)
            r.pages = [self.free_pages.pop() for _ in range(n_pages)]
            r.row = self.rows_free.pop()
            reqs.append(r)
        return reqs

    def release(self, reqs: list[Request]) -> None:
        for r in reqs:
            self.free_pages.extend(r.pages)
            self.rows_free.append(r.row)
            r.pages, r.row = [], -1

    # ---- prefill -------------------------------------------------------------------------------
    def prefill(self, reqs: list[Request]) -> None:
        """Prefills requests in packed chunks; appends each request's first token.
        Under expert parallelism every rank runs the same number of chunks
        (padding with one-token chunks) so the exchange steps line up."""
        pb = self.prefill_buf
        chunks, i = [], 0
        while i < len(reqs):
            chunk, ntok = [], 0
            while i < len(reqs) and len(chunk) < pb.max_seqs and ntok + len(reqs[i].prompt) <= pb.max_tokens:
                chunk.append(reqs[i])
                ntok += len(reqs[i].prompt)
                i += 1
            if not chunk:
                raise ValueError("prompt longer than max_prefill_tokens")
            chunks.append(chunk)
        n = self._max_over_ranks(len(chunks)) if self.ep is not None else len(chunks)
        from ..utils.trace import phase

        with phase("foundry.prefill"):
            for c in chunks:
                self._prefill_chunk(c)
        for _ in range(n - len(chunks)):
            pad = Request(rid=-1, prompt=[0], max_new_tokens=1, pages=[0])
            self._prefill_chunk([pad])

    def _max_over_ranks(self, v: int) -> int:
        import torch.distributed as dist

        dev = self.device if dist.get_backend() == "nccl" else "cpu"
        t = torch.tensor([v], dtype=torch.int64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return int(t.item())

    def _prefill_chunk(self, chunk: list[Request]) -> None:
        pb = self.prefill_buf
        off, seqlens = 0, []
        pb.h_cu[0] = 0
        for j, r in enumerate(chunk):
            n = len(r.prompt)
            pb.h_ids[off:off + n] = torch.tensor(r.prompt, dtype=torch.int32)
            pos = torch.arange(n, dtype=torch.int32)
            pb.h_pos[off:off + n] = pos
            pages = torch.tensor(r.pages, dtype=torch.int32)
            pb.h_slots[off:off + n] = pages[pos // PAGE] * PAGE + pos % PAGE
            off += n
            pb.h_cu[j + 1] = off
            pb.h_last[j] = off - 1
            seqlens.append(n)
        ts, tst = prefill_tiles(seqlens, PREFILL_TILE[PREFILL_IMPL])
        pb.h_tile_seq[:len(ts)] = torch.tensor(ts, dtype=torch.int32)
        pb.h_tile_start[:len(ts)] = torch.tensor(tst, dtype=torch.int32)
        n_seq = len(chunk)
        pb.input_ids[:off].copy_(pb.h_ids[:off], non_blocking=True)
        pb.positions[:off].copy_(pb.h_pos[:off], non_blocking=True)
        pb.slots[:off].copy_(pb.h_slots[:off], non_blocking=True)
        pb.cu_seqlens[:n_seq + 1].copy_(pb.h_cu[:n_seq + 1], non_blocking=True)
        pb.last_rows[:n_seq].copy_(pb.h_last[:n_seq], non_blocking=True)
        nt = len(ts)
        tile_seq = pb.tile_seq[:nt]
        tile_start = pb.tile_start[:nt]
        tile_seq.copy_(pb.h_tile_seq[:nt], non_blocking=True)
        tile_start.copy_(pb.h_tile_start[:nt], non_blocking=True)
        pb.num_tokens, pb.num_seqs = off, n_seq
        saved = (pb.tile_seq, pb.tile_start)
        pb.tile_seq, pb.tile_start = tile_seq, tile_start
        try:
            self.model.prefill(pb)
        finally:
            pb.tile_seq, pb.tile_start = saved
        pb.h_next[:n_seq].copy_(pb.next_ids[:n_seq])
        for j, r in enumerate(chunk):
            r.output.append(int(pb.h_next[j]))

    # ---- decode --------------------------------------------------------------------------------
    def bucket(self, n: int) -> int:
        for s in self.graph_sizes:
            if s >= n:
                return s
        raise ValueError(f"batch {n} exceeds the largest decode graph {self.graph_sizes[-1]}")

    def start_decode(self, reqs: list[Request]) -> int:
        """Lays the requests out in decode rows 0..n-1 and uploads their state."""
        st = self.state
        self.running = list(reqs)
        n = len(reqs)
        b = self.bucket(n)
        self.h_active[:b] = 0
        self.h_lens[:b] = 0
        self.h_tables[:b] = 0
        for j, r in enumerate(reqs):
            r.row = j
            self.h_tables[j, :len(r.pages)] = torch.tensor(r.pages, dtype=torch.int32)
            self.h_lens[j] = len(r.prompt) + len(r.output) - 1  # tokens already in the cache
            self.h_active[j] = 1
            self.h_in[j] = r.output[-1]
        st.block_tables[:b].copy_(self.h_tables[:b], non_blocking=True)
        st.seq_lens[:b].copy_(self.h_lens[:b], non_blocking=True)
        st.active[:b].copy_(self.h_active[:b], non_blocking=True)
        st.input_ids[:b].copy_(self.h_in[:b], non_blocking=True)
        return b

    def decode_step(self, b: int, use_graph: bool = True, sync_tokens: bool = True) -> torch.Tensor:
        """One decode step over rows [:b]: H2D of the step's input tokens, one
        graph launch, D2H of the sampled tokens."""
        st = self.state
        st.input_ids[:b].copy_(self.h_in[:b], non_blocking=True)
        if use_graph and b in self.graphs:
            self.graphs[b].replay()
        else:
            self._decode_body(b)
        if self.materialize_after_first_step:
            self.materialize_after_first_step = False
            self.materialize_graphs(background=True)
        self.h_out[:b].copy_(st.next_ids[:b], non_blocking=True)
        if sync_tokens:
            torch.cuda.current_stream().synchronize()
            self.h_in[:b] = self.h_out[:b]
        return self.h_out[:b]

    def _decode_body(self, b: int) -> None:
        from ..ops import _rt

        st = self.state
        # Padding rows are inactive: no cache writes, no attention. Kernels
        # start under programmatic dependent launch (set-up and weight loads
        # overlap the previous kernel).
        with _rt.pdl():
            self.model.decode(st, b)

    def generate(self, prompts: list[list[int]], max_new_tokens: int) -> list[list[int]]:
        reqs = self.add_requests(prompts, max_new_tokens)
        self.prefill(reqs)
        b = self.start_decode(reqs)
        steps = max_new_tokens - 1
        if self.ep is not None:  # every rank takes the same decode steps (and graph sizes stay per rank)
            steps = self._max_over_ranks(steps)
        for _ in range(steps):
            toks = self.decode_step(b)
            for r in reqs:
                if not r.done:
                    r.output.append(int(toks[r.row]))
        self.release(reqs)
        return [r.output for r in reqs]

    # ---- graphs --------------------------------------------------------------------------------
    def warmup(self) -> None:
        """Loads every kernel once (eagerly) so capture launches no first-use work."""
        st = self.state
        saved = st.active[:1].clone()
        st.active[:1].zero_()
        self.model.decode(st, 1)
        st.active[:1].copy_(saved)
        torch.cuda.synchronize()

    def capture_graphs(self, sizes: list[int] | None = None) -> float:
        from ..graphs import CUDAGraph, graph

        sizes = sizes or self.graph_sizes
        self.warmup()
        t0 = time.perf_counter()
        stream = torch.cuda.Stream()
        for s in sizes:
            g = CUDAGraph()
            with graph(g, stream=stream):
                self._decode_body(s)
            self.graphs[s] = g
        torch.cuda.synchronize()
        return time.perf_counter() - t0

    def materialize_graphs(self, sizes: list[int] | None = None, background: bool = True):
        """Gives restored decode graphs their own executables (largest batch
        first); with ``background`` on a daemon thread, returned. Graphs that
        are not restored ones (captured here) are skipped."""
        order = sorted(sizes if sizes is not None else list(self.graphs), reverse=True)

        def run():
            for s in order:
                if self._stop_materializing:
                    return
                g = self.graphs.get(s)
                if g is not None and hasattr(g, "materialize"):
                    g.materialize()

        if not background:
            run()
            return None
        self.wait_materialized()
        self._materializer = threading.Thread(target=run, name="foundry-materialize", daemon=True)
        self._materializer.start()
        return self._materializer

    def wait_materialized(self) -> None:
        """Blocks until a background materialisation (if any) has finished."""
        if self._materializer is not None:
            self._materializer.join()
            self._materializer = None

    def close(self) -> None:
        """Drops the decode graphs and unmaps the tensor-parallel buffers (graphs
        that reference the symmetric memory go first)."""
        self._stop_materializing = True
        self.wait_materialized()
        torch.cuda.synchronize()
        self.graphs.clear()
        if self.tp is not None:
            self.tp.close()
            self.tp = None
        if self.ep is not None:
            self.ep.close()
            self.ep = None
