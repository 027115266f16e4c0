"""Dense decoder (Llama-3 family) on foundry_b200's own kernels.

Weights use the nn.Linear layout ([out, in]); q/k/v projections are fused into
one [ (Hq + 2 Hkv) * 128, H ] matrix and gate/up into one [2 I, H] matrix, so a
layer is 4 GEMMs. Per decode step and layer the kernels are:

    rmsnorm -> GEMM(qkv) -> rope+kv-write -> decode-attention(+combine)
    -> GEMM(o, += residual) -> rmsnorm -> GEMM(gate_up) -> silu*mul
    -> GEMM(down, += residual)

Everything a step touches lives in the runner's static arena, so a decode
step is capturable as a CUDA graph and restorable in a fresh process.
``reference_forward`` is a plain fp32 PyTorch implementation used as the
numerics oracle in tests.
"""

from __future__ import annotations

import math
from dataclasses import asdict, dataclass, field

import torch

from .. import ops


@dataclass
class LlamaConfig:
    name: str = "llama-3-8b"
    hidden: int = 4096
    layers: int = 32
    n_q: int = 32
    n_kv: int = 8
    head_dim: int = 128
    inter: int = 14336
    vocab: int = 128256
    eps: float = 1e-5
    rope_theta: float = 500000.0
    rope_scaling: dict | None = None
    qk_norm: bool = False  # Qwen3-style per-head RMSNorm on q and k
    tie_embeddings: bool = False
    init_std: float = 0.02
    extra: dict = field(default_factory=dict)
    arch: str = "llama"

    @property
    def qkv_dim(self) -> int:
        return (self.n_q + 2 * self.n_kv) * self.head_dim

    def num_params(self) -> int:
        h, i = self.hidden, self.inter
        per_layer = h * self.qkv_dim + self.n_q * self.head_dim * h + 2 * h * i + i * h + 2 * h
        emb = self.vocab * h * (1 if self.tie_embeddings else 2)
        return self.layers * per_layer + emb + h

    def to_dict(self) -> dict:
        return asdict(self)


def llama3_8b() -> LlamaConfig:
    return LlamaConfig()


def llama3_70b() -> LlamaConfig:
    return LlamaConfig(name="llama-3-70b", hidden=8192, layers=80, n_q=64, n_kv=8, inter=28672)


def tiny(layers: int = 2, vocab: int = 4096) -> LlamaConfig:
    """Small config with the Llama-3-8B per-layer shapes (tests, smoke)."""
    return LlamaConfig(name=f"llama-3-8b-{layers}l", layers=layers, vocab=vocab)


def toy() -> LlamaConfig:
    return LlamaConfig(name="toy", hidden=512, layers=2, n_q=8, n_kv=2, inter=1024, vocab=1024)


CONFIGS = {"llama-3-8b": llama3_8b, "llama-3-70b": llama3_70b}

# Tensor parallel: row counts from which the row-parallel GEMM outputs are
# summed by an NVLS reduce-scatter + multicast instead of the slot exchange.
NVLS_MIN_ROWS = 128
NVLS_MIN_ROWS_2 = 512  # at 2 ranks (measured: slots faster at 256 rows, NVLS at 1024)
# "auto": from those row counts, at 2 ranks the GEMM all-reduces in its own
# epilogue (tiles reduced in the switch as they finish: fb_gemm_bf16_ar_bn*)
# and at more ranks the separate NVLS reduce kernel runs; below them the slot
# exchange. Measured on the Llama-3-70B down projection (profile_comm; us,
# slots / NVLS / fused): 2 ranks, 64 rows 83.5 / 93.0 / 105.6, 256 rows
# 97.0 / 109.4 / 120.0, 1024 rows 383.3 / 262.1 / 247.7; 8 ranks, 64 rows
# 43.8 / 41.8 / 56.6, 256 rows 87.0 / 53.2 / 68.5, 1024 rows 871.1 / 118.9 /
# 137.1 (at 8 ranks each CTA waits for eight ranks' tiles and reduces only an
# eighth of each). "nvls": the NVLS kernel from NVLS_MIN_ROWS rows at any rank
# count (tests); "fused": the fused kernel for every row count.
_TP_REDUCE = __import__("os").environ.get("FOUNDRY_TP_REDUCE", "auto")


class LlamaWeights:
    """All parameters (this rank's tensor-parallel shard), allocated from an
    arena and initialised deterministically.

    Tensor parallel layout (tp_size > 1): q/k/v and gate/up are split by output
    rows (heads / intermediate features, column parallel), o and down by input
    columns (row parallel: their outputs are partial sums), lm_head by vocab
    rows; the embedding table and the norms are replicated.
    """

    def __init__(self, cfg: LlamaConfig, arena, seed: int = 0, init: bool = True, tp_rank: int = 0,
                 tp_size: int = 1):
        self.cfg = cfg
        self.tp_rank, self.tp_size = tp_rank, tp_size
        for name, v in (("n_q", cfg.n_q), ("n_kv", cfg.n_kv), ("inter", cfg.inter), ("vocab", cfg.vocab)):
            if v % tp_size:
                raise ValueError(f"{name}={v} is not divisible by tp={tp_size}")
        self.nq_l, self.nkv_l = cfg.n_q // tp_size, cfg.n_kv // tp_size
        self.inter_l, self.vocab_l = cfg.inter // tp_size, cfg.vocab // tp_size
        h, d = cfg.hidden, cfg.head_dim
        self.qkv_dim_l = (self.nq_l + 2 * self.nkv_l) * d
        self.embed = arena.empty((cfg.vocab, h))
        self.layers = []
        for _ in range(cfg.layers):
            lw = {
                "attn_norm": arena.empty((h,)),
                "qkv": arena.empty((self.qkv_dim_l, h)),
                "o": arena.empty((h, self.nq_l * d)),
                "mlp_norm": arena.empty((h,)),
                "gate_up": arena.empty((2 * self.inter_l, h)),
                "down": arena.empty((h, self.inter_l)),
            }
            if cfg.qk_norm:
                lw["q_norm"] = arena.empty((d,))
                lw["k_norm"] = arena.empty((d,))
            self.layers.append(lw)
        self.final_norm = arena.empty((h,))
        if cfg.tie_embeddings and tp_size == 1:
            self.lm_head = self.embed
        else:
            self.lm_head = arena.empty((self.vocab_l, h))
        if init:
            self.init(seed)

    @property
    def vocab_offset(self) -> int:
        return self.tp_rank * self.vocab_l

    def shard_of(self, name: str, full: torch.Tensor) -> torch.Tensor:
        """The rows/columns of a full (unsharded) parameter that this rank holds."""
        cfg, r, d = self.cfg, self.tp_rank, self.cfg.head_dim
        key = name.split(".")[-1]
        if self.tp_size == 1 or key in ("attn_norm", "mlp_norm", "q_norm", "k_norm") or name in ("embed", "final_norm"):
            return full
        if key == "qkv":
            q = full[r * self.nq_l * d:(r + 1) * self.nq_l * d]
            k0 = cfg.n_q * d
            k = full[k0 + r * self.nkv_l * d:k0 + (r + 1) * self.nkv_l * d]
            v0 = (cfg.n_q + cfg.n_kv) * d
            v = full[v0 + r * self.nkv_l * d:v0 + (r + 1) * self.nkv_l * d]
            return torch.cat([q, k, v])
        if key == "gate_up":
            g = full[r * self.inter_l:(r + 1) * self.inter_l]
            u = full[cfg.inter + r * self.inter_l:cfg.inter + (r + 1) * self.inter_l]
            return torch.cat([g, u])
        if key == "o":
            return full[:, r * self.nq_l * d:(r + 1) * self.nq_l * d]
        if key == "down":
            return full[:, r * self.inter_l:(r + 1) * self.inter_l]
        if name == "lm_head":
            return full[r * self.vocab_l:(r + 1) * self.vocab_l]
        raise KeyError(name)

    def load_full(self, full: dict[str, torch.Tensor]) -> None:
        """Copies this rank's shard of each full parameter (e.g. a checkpoint)."""
        for name, t in self.tensors():
            t.copy_(self.shard_of(name, full[name]).to(device=t.device, dtype=t.dtype))

    def tensors(self):
        yield "embed", self.embed
        for i, lw in enumerate(self.layers):
            for k, v in lw.items():
                yield f"layers.{i}.{k}", v
        yield "final_norm", self.final_norm
        if self.lm_head is not self.embed:
            yield "lm_head", self.lm_head

    def init(self, seed: int) -> None:
        """Random init N(0, init_std) for matrices, ones for norm weights.
        Replicated tensors get the same values on every rank, shards differ."""
        for idx, (name, t) in enumerate(self.tensors()):
            if t.dim() == 1:
                ops.fill_(t, 1.0)
            else:
                rank_salt = 0 if name == "embed" else self.tp_rank * 7_919
                s = (seed * 1_000_003 + idx + rank_salt * 104_729) & ((1 << 63) - 1)
                ops.init_normal_(t, seed=s, std=self.cfg.init_std)


class LlamaModel:
    """Forward passes over preallocated buffers (no allocation inside a step)."""

    def __init__(self, cfg: LlamaConfig, weights: LlamaWeights, cos_sin: torch.Tensor):
        self.cfg = cfg
        self.w = weights
        self.cos_sin = cos_sin
        self.scale = 1.0 / math.sqrt(cfg.head_dim)

    # ---- one decode step for B sequences (graph-capturable) -------------------------------
    def decode(self, st, b: int) -> None:
        """``st`` is a DecodeState (runner/engine.py) with static buffers; uses rows [:b].

        With tensor parallelism (``st.tp`` set) the row-parallel o/down GEMMs
        multicast their tiles into the slot exchange and the next norm sums the
        ranks' slots (fused all-reduce); the lm_head is vocab-sharded."""
        cfg, w = self.cfg, self.w
        ops.decode_advance(st.seq_lens[:b], st.positions[:b], st.slots[:b], st.block_tables[:b], st.page,
                           st.active[:b])
        h = st.hidden[:b]
        x = st.normed[:b]
        ops.embedding(st.input_ids[:b], w.embed, h)
        self._begin(st, b)
        splits = st.attn_splits[b]
        pending = None  # output of the previous down-projection not yet added to h
        for li, lw in enumerate(w.layers):
            self._norm(st, pending, h, lw["attn_norm"], x, b)
            qkv = self._qkv(st, x, lw, b)
            ops.rope_kv_write(qkv, st.positions[:b], self.cos_sin, st.q[:b], st.k_cache[li], st.v_cache[li],
                              st.slots[:b], w.nq_l, w.nkv_l, lw.get("q_norm"), lw.get("k_norm"), cfg.eps)
            ops.decode_attention(st.q[:b], st.k_cache[li], st.v_cache[li], st.block_tables[:b], st.seq_lens[:b],
                                 st.attn_out[:b].view(b, w.nq_l, cfg.head_dim), st.max_pages, st.attn_ws,
                                 scale=self.scale, splits=splits)
            o = self._o_proj(st, st.attn_out[:b], lw, h, b)
            self._norm(st, o, h, lw["mlp_norm"], x, b)
            pending = self._mlp(st, x, h, lw, b)
        self._norm(st, pending, h, w.final_norm, x, b)
        ops.linear(x, w.lm_head, out=st.logits[:b], streamk=st.sk)
        if st.tp:
            from ..parallel import comm

            comm.argmax_sharded(st.tp.symm, st.logits[:b], w.vocab_offset, st.tp.pairs_offset, st.next_ids[:b])
        else:
            ops.argmax(st.logits[:b], st.next_ids[:b])

    # ---- per-layer pieces (overridden by other model families) ---------------------------
    def _begin(self, st, rows) -> None:
        """Per-forward setup shared by every layer (nothing for the dense bf16 model)."""

    def _qkv(self, st, x, lw, rows):
        return ops.linear(x, lw["qkv"], out=st.qkv[:rows], partials=getattr(st, "part", None))

    def _o_proj(self, st, inp, lw, h, rows):
        return self._row_parallel(st, inp, lw["o"], h, rows, which=0)

    def _mlp(self, st, x, h, lw, rows):
        """SwiGLU FFN of x; returns the pending output that the next norm adds into h."""
        # decode batches: one GEMM whose epilogue applies SiLU(gate) * up
        if ops.linear_swiglu(x, lw["gate_up"], st.act[:rows], sk=getattr(st, "swiglu_sk", None)) is None:
            gu = ops.linear(x, lw["gate_up"], out=st.gate_up[:rows], streamk=getattr(st, "sk", None))
            ops.silu_mul(gu, st.act[:rows])
        return self._row_parallel(st, st.act[:rows], lw["down"], h, rows, which=1)

    def _row_parallel(self, st, inp, weight, h, rows, which):
        """o / down projection. TP: multicast into the slot exchange + barrier and
        return ("slots", which); single GPU: residual epilogue (returns None) or
        split-K slices (returns the Partial)."""
        if st.tp:
            from ..parallel import comm

            ex = st.tp.slots
            many = ex.symm.multicast and (rows >= NVLS_MIN_ROWS_2 or (rows >= NVLS_MIN_ROWS and (
                ex.symm.world > 2 or _TP_REDUCE == "nvls")))
            fused = _TP_REDUCE == "fused" or (_TP_REDUCE == "auto" and many and ex.symm.world == 2)
            if fused and ex.gemm_allreduce(inp, weight, which):
                # one kernel: GEMM tiles reduced in the switch and multicast as they finish
                return ("reduced", which)
            if many:
                # many rows: partial sums reduced in the switch (one copy of the
                # output crosses NVLink per rank instead of world - 1)
                ops.linear(inp, weight, out=ex.slot(which, 0)[:rows])
                ex.nvls_reduce(which, rows)
                return ("reduced", which)
            target = ex.gemm_target(which)
            if target:
                ops.linear_multicast(inp, weight, target)
            else:
                ops.linear(inp, weight, out=ex.local_slot(which)[:rows])
                ex.broadcast_local_slot(which, rows)
            comm.barrier(st.tp.symm)
            return ("slots", which)
        r = ops.linear(inp, weight, out=h, residual=h, partials=getattr(st, "part", None))
        return r if isinstance(r, ops.Partial) else None

    def _norm(self, st, pending, h, weight, x, rows) -> None:
        """x = rmsnorm(h), first adding the pending projection output into h."""
        if pending is None:
            ops.rmsnorm(h, weight, x, self.cfg.eps)
        elif callable(pending):
            pending(weight, x)
        elif isinstance(pending, tuple):
            from ..parallel import comm

            slots = st.tp.slots.local_slots(pending[1])
            if pending[0] == "reduced":
                slots = slots[1:2]  # the reduced sum
            comm.add_rmsnorm_slots(slots, rows, h, weight, x, self.cfg.eps)
        else:
            ops.add_rmsnorm_partials(pending, h, weight, x, self.cfg.eps)

    # ---- prefill of a packed batch of prompts (eager) --------------------------------------
    def prefill(self, pb) -> None:
        """``pb`` is a PrefillBatch (runner/engine.py): packed ids, positions,
        slots, cu_seqlens, tile tables and scratch buffers; writes KV into the
        cache and the greedy next token of every prompt into pb.next_ids."""
        cfg, w = self.cfg, self.w
        t = pb.num_tokens
        h, x = pb.hidden[:t], pb.normed[:t]
        ops.embedding(pb.input_ids[:t], w.embed, h)
        nqd = w.nq_l * cfg.head_dim
        nkvd = w.nkv_l * cfg.head_dim
        self._begin(pb, t)
        pending = None
        for li, lw in enumerate(w.layers):
            self._norm(pb, pending, h, lw["attn_norm"], x, t)
            qkv = self._qkv(pb, x, lw, t)
            # Rotated q -> pb.q; rotated k and v -> paged cache and packed pb.k_rot / pb.v_rot.
            ops.rope_kv_write(qkv, pb.positions[:t], self.cos_sin, pb.q[:t], pb.k_cache[li], pb.v_cache[li],
                              pb.slots[:t], w.nq_l, w.nkv_l, lw.get("q_norm"), lw.get("k_norm"), cfg.eps,
                              k_out=pb.k_rot[:t], v_out=pb.v_rot[:t])
            from ..runner.engine import PREFILL_IMPL

            ops.prefill_attention(pb.q[:t].view(t, nqd), pb.k_rot[:t].view(t, nkvd), pb.v_rot[:t].view(t, nkvd),
                                  pb.attn_out[:t], pb.cu_seqlens, pb.tile_seq, pb.tile_start, w.nq_l, w.nkv_l,
                                  scale=self.scale, impl=PREFILL_IMPL)
            o = self._o_proj(pb, pb.attn_out[:t], lw, h, t)
            self._norm(pb, o, h, lw["mlp_norm"], x, t)
            pending = self._mlp(pb, x, h, lw, t)
        if pending is not None:
            # fold the last FFN output into h (the final norm runs on gathered rows)
            self._norm(pb, pending, h, w.final_norm, x, t)
        # last token of every prompt -> logits -> greedy token
        n = pb.num_seqs
        last = pb.last_rows[:n]
        torch.index_select(h, 0, last, out=pb.last_hidden[:n])
        ops.rmsnorm(pb.last_hidden[:n], w.final_norm, pb.last_normed[:n], cfg.eps)
        ops.linear(pb.last_normed[:n], w.lm_head, out=pb.logits[:n])
        if pb.tp:
            from ..parallel import comm

            comm.argmax_sharded(pb.tp.symm, pb.logits[:n], w.vocab_offset, pb.tp.pairs_offset, pb.next_ids[:n])
        else:
            ops.argmax(pb.logits[:n], pb.next_ids[:n])


# ---- fp32 reference (tests) --------------------------------------------------------------

def _rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _rope(x, pos, cos_sin):
    # x: [T, H, 128]; half rotation
    cs = cos_sin[pos]  # [T, 64, 2]
    c, s = cs[..., 0][:, None, :], cs[..., 1][:, None, :]
    x1, x2 = x[..., :64], x[..., 64:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def reference_forward(cfg: LlamaConfig, weights: LlamaWeights, ids: torch.Tensor, cos_sin: torch.Tensor,
                      layers: int | None = None) -> torch.Tensor:
    """fp32 causal forward of one sequence; returns logits [T, vocab]."""
    f = lambda t: t.float()  # noqa: E731
    t_len = ids.numel()
    pos = torch.arange(t_len, device=ids.device)
    h = f(weights.embed)[ids.long()]
    d = cfg.head_dim
    g = cfg.n_q // cfg.n_kv
    for lw in weights.layers[: layers or cfg.layers]:
        x = _rms(h, f(lw["attn_norm"]), cfg.eps)
        qkv = x @ f(lw["qkv"]).T
        q = qkv[:, : cfg.n_q * d].view(t_len, cfg.n_q, d)
        k = qkv[:, cfg.n_q * d: (cfg.n_q + cfg.n_kv) * d].view(t_len, cfg.n_kv, d)
        v = qkv[:, (cfg.n_q + cfg.n_kv) * d:].view(t_len, cfg.n_kv, d)
        if cfg.qk_norm:
            q = _rms(q, f(lw["q_norm"]), cfg.eps)
            k = _rms(k, f(lw["k_norm"]), cfg.eps)
        q, k = _rope(q, pos, cos_sin), _rope(k, pos, cos_sin)
        k = k.repeat_interleave(g, dim=1)
        v = v.repeat_interleave(g, dim=1)
        att = torch.einsum("thd,shd->hts", q, k) / math.sqrt(d)
        mask = torch.triu(torch.ones(t_len, t_len, dtype=torch.bool, device=ids.device), 1)
        att = att.masked_fill(mask, float("-inf")).softmax(-1)
        o = torch.einsum("hts,shd->thd", att, v).reshape(t_len, cfg.n_q * d)
        h = h + o @ f(lw["o"]).T
        x = _rms(h, f(lw["mlp_norm"]), cfg.eps)
        gu = x @ f(lw["gate_up"]).T
        gate, up = gu[:, : cfg.inter], gu[:, cfg.inter:]
        h = h + (torch.nn.functional.silu(gate) * up) @ f(lw["down"]).T
    x = _rms(h, f(weights.final_norm), cfg.eps)
    return x @ f(weights.lm_head).T
