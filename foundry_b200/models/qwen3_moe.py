"""Qwen3-MoE decoder (Qwen3-30B-A3B shape) with block-scaled fp8 weights.

Per layer: RMSNorm -> QKV -> per-head q/k RMSNorm + RoPE + paged KV write
-> decode attention (GQA 32/4) -> O (+= residual) -> RMSNorm -> router
(bf16, 128 experts) -> softmax top-8 (renormalised) -> grouped fp8 expert
FFN (gate_up, SiLU*up, down) -> top-k weighted combine fused with the next
RMSNorm. The expert weights are e4m3 with 128 x 128 block scales and their
activations are quantised per token per 128 features right before each fp8
GEMM. The attention projections come from the same block-scaled fp8
checkpoint; by default they are dequantised once at load into bf16 and run
on the dense bf16 GEMM (split-K slices consumed by RoPE / the next norm,
residual epilogue), which at decode batch sizes is faster than the grouped
fp8 kernel for these 19 MB per layer; ``attn_fp8=True`` keeps them e4m3.

Expert parallelism (``ep_size`` > 1, with DP attention: every rank runs the
attention of its own sequences) shards the experts; the dispatch/combine
exchange runs over symmetric memory (foundry_b200.parallel.ep).

The reference serves this model through vLLM/SGLang with DeepEP + DeepGEMM
(reference recipe/vllm/serve_qwen3-30ba3b_ep.sh:48-70,
recipe/sglang/serve_qwen3-30ba3bfp8_ep.sh:51-70); this is our own engine.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from .. import ops
from ..ops import moe as M
from .llama import LlamaConfig, LlamaModel, _rms, _rope


@dataclass
class Qwen3MoeConfig(LlamaConfig):
    name: str = "qwen3-30b-a3b"
    hidden: int = 2048
    layers: int = 48
    n_q: int = 32
    n_kv: int = 4
    head_dim: int = 128
    inter: int = 0               # no dense FFN
    vocab: int = 151936
    eps: float = 1e-6
    rope_theta: float = 1000000.0
    qk_norm: bool = True
    num_experts: int = 128
    topk: int = 8
    moe_inter: int = 768
    norm_topk_prob: bool = True
    arch: str = "qwen3_moe"
    # fp8 GEMM flavour: "promote" = e4m3 x e4m3 tcgen05 kind::f8f6f4 with
    # per-128-K promotion (activations quantised per token per 128), "w8" =
    # e4m3 weights dequantised on chip, bf16 activations, kind::f16
    fp8_gemm: str = "promote"
    fp8_prefetch: int = 0  # L2 prefetch distance of weight tiles (k-blocks)
    # qkv / o projections kept as e4m3 block weights (True) or dequantised
    # once into bf16 (False: same values up to one bf16 rounding)
    attn_fp8: bool = False

    def num_params(self) -> int:
        h, d = self.hidden, self.head_dim
        attn = h * self.qkv_dim + self.n_q * d * h + 2 * d
        moe = self.num_experts * 3 * h * self.moe_inter + self.num_experts * h
        return self.layers * (attn + moe + 2 * h) + 2 * self.vocab * h + h

    def active_params(self) -> int:
        h, d = self.hidden, self.head_dim
        attn = h * self.qkv_dim + self.n_q * d * h
        return self.layers * (attn + self.topk * 3 * h * self.moe_inter + self.num_experts * h) + 2 * self.vocab * h


def qwen3_30b_a3b() -> Qwen3MoeConfig:
    return Qwen3MoeConfig()


def tiny_moe(layers: int = 2, vocab: int = 4096, experts: int = 32) -> Qwen3MoeConfig:
    """Small config with Qwen3-30B-A3B per-layer shapes except the expert count."""
    return Qwen3MoeConfig(name=f"qwen3-moe-{layers}l-{experts}e", layers=layers, vocab=vocab, num_experts=experts)


class Qwen3MoeWeights:
    """Parameters of one rank: attention replicated (DP attention), experts
    [ep_rank * E / ep, (ep_rank + 1) * E / ep) local."""

    def __init__(self, cfg: Qwen3MoeConfig, arena, seed: int = 0, init: bool = True, tp_rank: int = 0,
                 tp_size: int = 1, ep_rank: int = 0, ep_size: int = 1):
        if tp_size != 1:
            raise ValueError("Qwen3-MoE runs attention data-parallel; use ep_size, not tp")
        if cfg.num_experts % ep_size:
            raise ValueError(f"{cfg.num_experts} experts not divisible by ep={ep_size}")
        self.cfg = cfg
        self.tp_rank, self.tp_size = 0, 1
        self.ep_rank, self.ep_size = ep_rank, ep_size
        self.e_local = cfg.num_experts // ep_size
        self.e0 = ep_rank * self.e_local
        h, d = cfg.hidden, cfg.head_dim
        self.nq_l, self.nkv_l = cfg.n_q, cfg.n_kv
        self.inter_l, self.vocab_l = 0, cfg.vocab
        self.qkv_dim_l = cfg.qkv_dim
        self.embed = arena.empty((cfg.vocab, h))
        self.layers = []
        for _ in range(cfg.layers):
            self.layers.append({
                "attn_norm": arena.empty((h,)),
                "qkv": self._proj(arena, cfg.qkv_dim, h),
                "o": self._proj(arena, h, cfg.n_q * d),
                "q_norm": arena.empty((d,)),
                "k_norm": arena.empty((d,)),
                "mlp_norm": arena.empty((h,)),
                "router": arena.empty((cfg.num_experts, h)),
                "w13": M.Fp8Weight.empty(arena, self.e_local, 2 * cfg.moe_inter, h),
                "w2": M.Fp8Weight.empty(arena, self.e_local, h, cfg.moe_inter),
            })
        self.final_norm = arena.empty((h,))
        self.lm_head = arena.empty((cfg.vocab, h))
        if init:
            self.init(seed)

    vocab_offset = 0

    def _proj(self, arena, rows: int, cols: int):
        return M.Fp8Weight.empty(arena, 1, rows, cols) if self.cfg.attn_fp8 else arena.empty((rows, cols))

    def tensors(self):
        yield "embed", self.embed
        for i, lw in enumerate(self.layers):
            for k, v in lw.items():
                yield f"layers.{i}.{k}", v
        yield "final_norm", self.final_norm
        yield "lm_head", self.lm_head

    def init(self, seed: int) -> None:
        """N(0, init_std) matrices (fp8 ones quantised per block), ones for norms.
        Seeds depend only on the tensor, and expert shards draw their rows of
        the full expert matrix, so every EP degree sees the same model. bf16
        attention projections are the dequantised fp8 block weights that
        ``attn_fp8`` would hold."""
        std = self.cfg.init_std
        for idx, (name, t) in enumerate(self.tensors()):
            s = (seed * 1_000_003 + idx * 7_919) & ((1 << 63) - 1)
            if isinstance(t, M.Fp8Weight):
                expert = name.endswith(("w13", "w2"))  # expert shards draw their rows of the full matrix
                M.init_fp8_block_(t, s, std, row_offset=self.e0 * t.rows if expert else 0)
            elif name.endswith((".qkv", ".o")):
                rows, cols = t.shape
                tmp = M.Fp8Weight(torch.empty((rows, cols), dtype=torch.uint8, device=t.device),
                                  torch.zeros((1, rows // 128, M.kb_pad(cols // 128)), dtype=torch.float32,
                                              device=t.device), 1, rows, cols)
                M.init_fp8_block_(tmp, s, std)
                M.dequantize_block_fp8_(tmp, t)
            elif t.dim() == 1:
                ops.fill_(t, 1.0)
            else:
                ops.init_normal_(t, seed=s, std=std)


class Qwen3MoeModel(LlamaModel):
    """Decode / prefill of Qwen3-MoE on the shared attention path of LlamaModel."""

    # scratch buffers a DecodeState / PrefillBatch needs for `rows` tokens
    @staticmethod
    def buffers(cfg: Qwen3MoeConfig, w: Qwen3MoeWeights, rows: int) -> dict:
        h, d, k, i = cfg.hidden, cfg.head_dim, cfg.topk, cfg.moe_inter
        p = rows * k
        u8, f32, i32 = torch.uint8, torch.float32, torch.int32
        sr, kp = M.scale_rows, M.kb_pad
        dense = {
            "xq_h": ((rows, h), u8), "xs_h": ((sr(rows), kp(h // 128)), f32),
            "xq_o": ((rows, cfg.n_q * d), u8), "xs_o": ((sr(rows), kp(cfg.n_q * d // 128)), f32),
            "dchunks": ((rows // 32 + 1, 4), i32), "dmeta": ((4,), i32),
        } if cfg.attn_fp8 else {}
        return dense | {
            "rlogits": ((rows, cfg.num_experts), torch.bfloat16), "tids": ((rows, k), i32), "tw": ((rows, k), f32),
            "pos": ((p,), i32), "ecounts": ((cfg.num_experts,), i32),
            "chunks": ((M.max_chunks(p, w.e_local, 32), 4), i32), "meta": ((4,), i32),
            "mxq": ((p, h), u8), "mxs": ((sr(p), kp(h // 128)), f32),
            "y13": ((p, 2 * i), torch.bfloat16), "maq": ((p, i), u8), "mas": ((sr(p), kp(i // 128)), f32),
            "y2": ((p, h), torch.bfloat16),
            "mx16": ((p, h), torch.bfloat16), "act16": ((p, i), torch.bfloat16),
        }

    def __init__(self, cfg: Qwen3MoeConfig, weights: Qwen3MoeWeights, cos_sin: torch.Tensor):
        super().__init__(cfg, weights, cos_sin)
        import os

        self.kind = os.environ.get("FOUNDRY_FP8_GEMM", cfg.fp8_gemm)
        self.pf = int(os.environ.get("FOUNDRY_FP8_PREFETCH", cfg.fp8_prefetch))
        if self.kind not in ("promote", "w8"):
            raise ValueError(f"fp8_gemm must be 'promote' or 'w8', got {self.kind!r}")

    def _bn_dense(self, rows: int) -> int:
        return 32 if rows <= 32 else 64

    def _bn_moe(self, pairs: int) -> int:
        # promote: 32-token tiles at three CTAs per SM beat 64-token tiles at
        # every decode size measured (512 to 1024 tokens, 64 or 128 experts)
        if self.kind == "promote":
            return 32
        return 64 if pairs > 32 * self.w.e_local else 32

    def _gemm(self, w, x, xq, xs, chunks, meta, out, units, bn, residual=None, stream=False):
        if self.kind == "w8":
            return M.gemm_w8(w, x, chunks, meta, out, max_units=units, bn=bn, residual=residual,
                             stream_weights=stream, prefetch=self.pf)
        return M.gemm_fp8(w, xq, xs, chunks, meta, out, max_units=units, bn=bn, residual=residual,
                          stream_weights=stream, prefetch=self.pf)

    def _begin(self, st, rows) -> None:
        if self.w.cfg.attn_fp8:
            M.dense_chunks(rows, self._bn_dense(rows), st.dchunks, st.dmeta)

    def _dense(self, st, x, xq, xs, w, out, rows, residual=None):
        if self.kind == "promote":
            M.quantize_rows(x, xq, xs)
        bn = self._bn_dense(rows)
        return self._gemm(w, x, xq, xs, st.dchunks, st.dmeta, out, math.ceil(rows / bn) * (w.rows // 128), bn,
                          residual=residual)

    def _qkv(self, st, x, lw, rows):
        if not isinstance(lw["qkv"], M.Fp8Weight):
            return super()._qkv(st, x, lw, rows)
        return self._dense(st, x, st.xq_h, st.xs_h, lw["qkv"], st.qkv[:rows], rows)

    def _o_proj(self, st, inp, lw, h, rows):
        if not isinstance(lw["o"], M.Fp8Weight):
            return super()._o_proj(st, inp, lw, h, rows)
        self._dense(st, inp, st.xq_o, st.xs_o, lw["o"], h, rows, residual=h)
        return None

    def _mlp(self, st, x, h, lw, rows):
        cfg, w = self.cfg, self.w
        k = cfg.topk
        p = rows * k
        ops.linear(x, lw["router"], out=st.rlogits[:rows])
        M.topk(st.rlogits[:rows], k, st.tids[:rows], st.tw[:rows], renorm=cfg.norm_topk_prob)
        if getattr(st, "ep", None) is not None:
            return st.ep.moe(self, st, x, h, lw, rows)
        bn = self._bn_moe(p)
        M.plan(st.tids, p, w.e_local, bn, st.pos, st.ecounts, st.chunks, st.meta)
        units = M.max_chunks(p, w.e_local, bn)
        if self.kind == "w8":
            M.scatter_rows(x, st.pos, k, st.mx16)
            self._gemm(lw["w13"], st.mx16, None, None, st.chunks, st.meta, st.y13, units * (2 * cfg.moe_inter // 128),
                       bn, stream=True)
            ops.silu_mul(st.y13[:p], st.act16[:p])
            self._gemm(lw["w2"], st.act16, None, None, st.chunks, st.meta, st.y2, units * (cfg.hidden // 128), bn,
                       stream=True)
        else:
            M.quantize_rows(x, st.mxq, st.mxs, pos=st.pos, topk=k)
            self._gemm(lw["w13"], None, st.mxq, st.mxs, st.chunks, st.meta, st.y13,
                       units * (2 * cfg.moe_inter // 128), bn, stream=True)
            M.silu_mul_quant(st.y13, p, st.maq, st.mas)
            self._gemm(lw["w2"], None, st.maq, st.mas, st.chunks, st.meta, st.y2, units * (cfg.hidden // 128), bn,
                       stream=True)

        def combine(norm_w, x_out, _st=st, _h=h, _k=k):
            M.combine_add_rmsnorm(_st.y2, _st.pos, _st.tw, _k, _h, norm_w, x_out, cfg.eps)

        return combine


def reference_forward(cfg: Qwen3MoeConfig, weights: Qwen3MoeWeights, ids: torch.Tensor, cos_sin: torch.Tensor,
                      layers: int | None = None) -> torch.Tensor:
    """fp32 causal forward of one sequence with the dequantised weights (no
    activation quantisation); returns logits [T, vocab]. Needs all experts
    local (ep_size 1)."""
    assert weights.ep_size == 1
    f = lambda t: t.dequant() if isinstance(t, M.Fp8Weight) else t.float()  # noqa: E731
    t_len = ids.numel()
    pos = torch.arange(t_len, device=ids.device)
    h = f(weights.embed)[ids.long()]
    d = cfg.head_dim
    g = cfg.n_q // cfg.n_kv
    e, i = cfg.num_experts, cfg.moe_inter
    for lw in weights.layers[: layers or cfg.layers]:
        x = _rms(h, f(lw["attn_norm"]), cfg.eps)
        qkv = x @ f(lw["qkv"]).T
        q = qkv[:, : cfg.n_q * d].view(t_len, cfg.n_q, d)
        k = qkv[:, cfg.n_q * d: (cfg.n_q + cfg.n_kv) * d].view(t_len, cfg.n_kv, d)
        v = qkv[:, (cfg.n_q + cfg.n_kv) * d:].view(t_len, cfg.n_kv, d)
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
        probs = (x @ f(lw["router"]).T).softmax(-1)
        tw, tid = probs.topk(cfg.topk, dim=-1)
        if cfg.norm_topk_prob:
            tw = tw / tw.sum(-1, keepdim=True)
        w13 = lw["w13"].dequant().view(e, 2 * i, cfg.hidden)
        w2 = lw["w2"].dequant().view(e, cfg.hidden, i)
        out = torch.zeros_like(h)
        for ex in tid.unique().tolist():
            rows, slot = (tid == ex).nonzero(as_tuple=True)
            gu = x[rows] @ w13[ex].T
            act = torch.nn.functional.silu(gu[:, :i]) * gu[:, i:]
            out.index_add_(0, rows, (act @ w2[ex].T) * tw[rows, slot, None])
        h = h + out
    x = _rms(h, f(weights.final_norm), cfg.eps)
    return x @ f(weights.lm_head).T


CONFIGS = {"qwen3-30b-a3b": qwen3_30b_a3b}
