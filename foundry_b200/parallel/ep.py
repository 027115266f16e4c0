"""Expert parallelism with data-parallel attention (Qwen3-MoE).

Every rank runs attention for its own sequences and owns E / world experts.
The token exchange of a MoE layer is three of our own kernels plus the
GEMMs, all over symmetric memory (identical peer addresses in every process,
so the captured graphs restore with valid peer pointers):

    fb_ep_count -> barrier -> fb_ep_plan -> fb_ep_dispatch (fused e4m3
    quantise + P2P store of each token row into its owners' receive
    buffers) -> barrier -> grouped GEMM gate_up -> silu*up (+quantise) ->
    grouped GEMM down whose epilogue stores each row into the source rank's
    combine buffer over NVLink -> barrier -> top-k weighted sum + residual +
    RMSNorm (fb_moe_combine_add_rmsnorm) on the source rank.

Every rank issues the same collective steps in the same order (the engine
pads prefill chunks and decode steps so that they match across ranks).

Parity: the reference persists DeepEP low-latency dispatch/combine over
NVSHMEM inside vLLM/SGLang graphs (reference tests/test_deepep_fabric.py:
319-379, python/foundry/integration/vllm/hooks.py:682-706); this is our own
exchange with the quantisation and the weighted sum fused in.
"""

from __future__ import annotations

import math

import torch

from ..ops import _rt
from ..ops import moe as M
from . import comm
from .symm import CTRL_BYTES, SymmetricMemory

_IMG = "moe"


def _align(n: int, a: int = 4096) -> int:
    return -(-n // a) * a


class EPContext:
    """Symmetric buffers of the expert exchange for up to ``max_tokens``
    tokens per rank and step."""

    def __init__(self, cfg, max_tokens: int, group=None):
        import torch.distributed as dist

        self.cfg = cfg
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.max_tokens = max_tokens
        e, k, h = cfg.num_experts, cfg.topk, cfg.hidden
        if e % self.world:
            raise ValueError(f"{e} experts not divisible by {self.world} ranks")
        self.e_local = e // self.world
        self.kbp = M.kb_pad(h // 128)
        self.max_recv = self.world * max_tokens * k
        off = CTRL_BYTES
        self.counts_off = off
        off = _align(off + self.world * e * 4)
        self.q_off = off
        off = _align(off + self.max_recv * h)
        self.s_off = off
        off = _align(off + M.scale_rows(self.max_recv) * self.kbp * 4)
        self.map_off = off
        off = _align(off + self.max_recv * 4)
        self.comb_off = off
        off = _align(off + max_tokens * k * h * 2)
        self.symm = SymmetricMemory(off, group)
        s = self.symm
        self.counts = s.tensor(s.rank, (self.world, e), torch.int32, self.counts_off)
        self.recv_q = s.tensor(s.rank, (self.max_recv, h), torch.uint8, self.q_off)
        self.recv_s = s.tensor(s.rank, (M.scale_rows(self.max_recv), self.kbp), torch.float32, self.s_off)
        self.rowmap = s.tensor(s.rank, (self.max_recv,), torch.int32, self.map_off)
        self.comb = s.tensor(s.rank, (max_tokens * k, h), torch.bfloat16, self.comb_off)
        self.recv_q.zero_()
        self.recv_s.zero_()
        self.comb.zero_()
        torch.cuda.synchronize()

    def close(self) -> None:
        self.symm.close()

    def buffers(self, rows: int) -> dict:
        """Per-state scratch (local memory) of one forward of ``rows`` tokens."""
        cfg = self.cfg
        k, i = cfg.topk, cfg.moe_inter
        r = self.world * rows * k
        i32, f32 = torch.int32, torch.float32
        return {
            "ep_dst": ((rows * k,), i32), "ep_chunks": ((M.max_chunks(r, self.e_local, 32), 4), i32),
            "ep_meta": ((4,), i32), "ep_y13": ((r, 2 * i), torch.bfloat16), "ep_aq": ((r, i), torch.uint8),
            "ep_as": ((M.scale_rows(r), M.kb_pad(i // 128)), f32), "ep_ident": ((rows * k,), i32),
        }

    def moe(self, model, st, x, h, lw, rows):
        """The MoE block of one layer for this rank's ``rows`` tokens (router
        top-k already in st.tids / st.tw). Returns the combine closure that
        the next norm calls."""
        cfg = self.cfg
        s = self.symm
        k, e = cfg.topk, cfg.num_experts
        p = rows * k
        r_max = self.world * rows * k
        bn = model._bn_moe(r_max // self.world)
        _rt.launch(_IMG, "fb_ep_count", (1,), (256,), [
            st.tids.data_ptr(), p, e, s.rank, s.world, s.base, s.stride, self.counts_off])
        comm.barrier(s)
        _rt.launch(_IMG, "fb_ep_plan", (1,), (1024,), [
            self.counts.data_ptr(), st.tids.data_ptr(), p, e, self.e_local, s.rank, s.world, bn,
            st.ep_dst.data_ptr(), st.ep_chunks.data_ptr(), st.ep_meta.data_ptr()])
        groups = math.ceil(cfg.hidden // 128 / 4)
        _rt.launch(_IMG, "fb_ep_dispatch", (math.ceil(rows * groups / 8),), (256,), [
            x.data_ptr(), x.stride(0), rows, cfg.hidden, st.tids.data_ptr(), st.ep_dst.data_ptr(), k, self.e_local,
            s.rank, s.base, s.stride, self.q_off, self.s_off, self.map_off])
        comm.barrier(s)
        units = M.max_chunks(r_max, self.e_local, bn)
        M.gemm_fp8(lw["w13"], self.recv_q, self.recv_s, st.ep_chunks, st.ep_meta, st.ep_y13,
                   max_units=units * (2 * cfg.moe_inter // 128), bn=bn, stream_weights=True)
        M.silu_mul_quant(st.ep_y13, r_max, st.ep_aq, st.ep_as, meta=st.ep_meta)
        M.gemm_fp8(lw["w2"], st.ep_aq, st.ep_as, st.ep_chunks, st.ep_meta, s.base + self.comb_off,
                   max_units=units * (cfg.hidden // 128), bn=bn, stream_weights=True, peer_rowmap=self.rowmap,
                   peer_stride=s.stride, ldo=cfg.hidden)
        comm.barrier(s)

        def combine(norm_w, x_out, _h=h, _st=st):
            M.combine_add_rmsnorm(self.comb, _st.ep_ident, _st.tw, k, _h, norm_w, x_out, cfg.eps)

        return combine


__all__ = ["EPContext"]
