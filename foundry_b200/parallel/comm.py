"""Collective ops on symmetric memory (csrc/kernels/comm.cu) and the slot
exchange used by the fused GEMM -> all-reduce of tensor-parallel layers.

Fused all-reduce of a row-parallel GEMM (TP):
    1. the GEMM epilogue multicasts each output tile into this rank's slot of
       every rank's slot buffer (``SlotExchange.gemm_target``: an NVLS
       multicast address, so the tile crosses NVLink once, as it is produced);
    2. ``barrier``: every rank's slot is complete everywhere;
    3. the consumer sums the world slots in rank order (deterministic) with the
       residual and applies RMSNorm (``add_rmsnorm_slots``).
Two slot buffers alternate so a fast rank never overwrites slots a slower
rank is still reading (the barrier between uses orders them).
"""

from __future__ import annotations

import math

import torch

from ..ops import _rt
from .symm import CTRL_BYTES, SymmetricMemory

_IMG = "comm"


def barrier(symm: SymmetricMemory) -> None:
    _rt.launch(_IMG, "fb_sym_barrier", (1,), (64,), [symm.base, symm.stride, symm.rank, symm.world])


def all_reduce(symm: SymmetricMemory, offset: int, n: int, out: torch.Tensor, algo: str = "oneshot") -> torch.Tensor:
    """Sum over ranks of the n bf16 values at ``offset`` of every rank's buffer
    into ``out`` (local). Includes the barrier that makes the inputs visible;
    the caller must not rewrite its input before the next barrier."""
    assert out.dtype == torch.bfloat16 and out.numel() >= n and n % 8 == 0
    barrier(symm)
    if algo == "nvls" and symm.multicast:
        # reduce a shard each, multicast it to every rank's out slot, barrier
        out_off = offset + n * 2
        _rt.launch(_IMG, "fb_allreduce_nvls_bf16", (min(132, math.ceil(n / 8 / 256)),), (256,),
                   [symm.mc_ptr + offset, symm.mc_ptr + out_off, n, symm.rank, symm.world])
        barrier(symm)
        out.view(-1)[:n].copy_(symm.tensor(symm.rank, (n,), torch.bfloat16, out_off))
        return out
    _rt.launch(_IMG, "fb_allreduce_oneshot_bf16", (min(4 * 148, max(1, math.ceil(n / 8 / 256))),), (256,),
               [symm.base, symm.stride, offset, out.data_ptr(), n, symm.world])
    return out


# Control block of the fused GEMM + all-reduce kernel (csrc/kernels/gemm_bf16.cu,
# fb_gemm_bf16_ar_bn*): epoch, exit ticket, done[2], ready[2][AR_MAX_TILES]
# (u32 words from word 16), one block per slot buffer.
AR_MAX_TILES = 4096
AR_BLOCK_BYTES = -(-((16 + 2 * AR_MAX_TILES) * 4) // 4096) * 4096


class SlotExchange:
    """Two alternating [world][rows][cols] bf16 slot buffers in symmetric
    memory, and (``ar_offset``) the two control blocks of the fused GEMM +
    all-reduce, zeroed by the owner before first use."""

    def __init__(self, symm: SymmetricMemory, offset: int, rows: int, cols: int, ar_offset: int | None = None):
        self.symm = symm
        self.rows, self.cols = rows, cols
        self.slot_bytes = rows * cols * 2
        self.buf_bytes = symm.world * self.slot_bytes
        self.offset = offset
        if offset + 2 * self.buf_bytes > symm.size:
            raise ValueError("symmetric buffer too small for the slot exchange")
        if ar_offset is not None and ar_offset + 2 * AR_BLOCK_BYTES > symm.size:
            raise ValueError("symmetric buffer too small for the all-reduce control blocks")
        self.ar_offset = ar_offset
        self.which = 0

    def gemm_allreduce(self, x: torch.Tensor, w: torch.Tensor, which: int) -> bool:
        """x @ w.T summed over ranks into slot 1 of buffer ``which`` on every
        rank, by one kernel: the GEMM epilogue writes this rank's partial tile
        into slot 0, and as soon as every rank has its tile the CTA reduces
        its 1/world share of the tile's rows in the switch and multicasts the
        sums (a tile-granular reduce-scatter + all-gather over NVSwitch that
        overlaps the next tile's MMAs). Returns False, launching nothing,
        when this buffer has no multicast object or control block, or the
        shape does not fit the kernel (then use another path)."""
        from ..ops import gemm as G

        s = self.symm
        t_tok, k = x.shape
        n_out = w.shape[0]
        if not s.multicast or self.ar_offset is None or t_tok > self.rows or n_out != self.cols or n_out % 8:
            return False
        p = G.plan(t_tok, n_out, k, allow_split=False, allow_pair=False)
        units = math.ceil((n_out if p.swap else t_tok) / G.BM) * math.ceil((t_tok if p.swap else n_out) / p.bn)
        if units > AR_MAX_TILES:
            return False
        part = self.slot(which, 0)[:t_tok]
        if p.swap:
            a, b, mg, ng = w, x, n_out, t_tok
            om = G.out_maps(part.data_ptr(), 0, n_out, t_tok, part.stride(0), p.bn)
            if om is None:
                return False
            mode = G.EPI_TRANSPOSE | G.EPI_TMA_OUT
            if math.ceil(ng / p.bn) == 1:
                mode |= G.EPI_A_STREAM
            if _rt.pdl_active():
                mode |= G.EPI_A_CONST
            omap = om[0]
        else:
            a, b, mg, ng, mode, omap = x, w, t_tok, n_out, 0, G._NO_MAP
        mode |= (min(p.pf, 255) & 0xFF) << 8
        p_mc = s.mc_ptr + self._buf_off(which)
        fl = self.ar_offset + which * AR_BLOCK_BYTES
        _rt.launch("gemm_bf16", f"fb_gemm_bf16_ar_bn{p.bn}", (min(units, _rt.sm_count()),), (192,), [
            G.tmap(a, G.BM), G.tmap(b, p.bn), omap, part.data_ptr(), mg, ng, k, part.stride(0), mode,
            p_mc, p_mc + self.slot_bytes, s.ptr(s.rank, fl), s.mc_ptr + fl, s.rank, s.world,
        ], smem=G.smem_bytes(p.bn, 1))
        return True

    @property
    def nbytes(self) -> int:
        return 2 * self.buf_bytes

    def _buf_off(self, which: int) -> int:
        return self.offset + which * self.buf_bytes

    def gemm_target(self, which: int) -> int:
        """Multicast address of this rank's slot (GEMM output with EPI_MCAST), or
        0 when the node has no multicast (then use ``local_slot`` + broadcast)."""
        s = self.symm
        if not s.multicast:
            return 0
        return s.mc_ptr + self._buf_off(which) + s.rank * self.slot_bytes

    def local_slots(self, which: int) -> torch.Tensor:
        s = self.symm
        return s.tensor(s.rank, (s.world, self.rows, self.cols), torch.bfloat16, self._buf_off(which))

    def local_slot(self, which: int) -> torch.Tensor:
        return self.local_slots(which)[self.symm.rank]

    def slot(self, which: int, i: int) -> torch.Tensor:
        """Slot ``i`` of buffer ``which`` in this rank's memory ([rows, cols])."""
        return self.local_slots(which)[i]

    def nvls_reduce(self, which: int, rows: int) -> None:
        """Large-row alternative to the slot exchange (same buffers): every rank
        has written its partial GEMM output into slot 0 of buffer ``which`` (the
        same offset on every rank); after a barrier each rank reduces 1/world
        of it in the switch (multimem.ld_reduce, fp32 accumulation) and
        multicasts the sum into slot 1 of every rank; a second barrier makes
        slot 1 complete everywhere. NVLink ingress per rank: one copy of the
        output instead of world - 1 copies."""
        s = self.symm
        n = rows * self.cols
        barrier(s)
        mc_in = s.mc_ptr + self._buf_off(which)
        _rt.launch(_IMG, "fb_allreduce_nvls_bf16", (min(132, max(1, math.ceil(n / 8 / 256))),), (256,),
                   [mc_in, mc_in + self.slot_bytes, n, s.rank, s.world])
        barrier(s)

    def broadcast_local_slot(self, which: int, rows: int) -> None:
        """No-multicast fallback: copy this rank's slot to every rank over P2P."""
        s = self.symm
        nbytes = rows * self.cols * 2
        _rt.launch(_IMG, "fb_sym_broadcast", (min(4 * 148, max(1, math.ceil(nbytes / 16 / 256))),), (256,), [
            self.local_slot(which).data_ptr(), s.base, s.stride, self._buf_off(which) + s.rank * self.slot_bytes,
            nbytes, s.world])


def add_rmsnorm_slots(slots: torch.Tensor, rows: int, h: torch.Tensor, w: torch.Tensor, x: torch.Tensor,
                      eps: float) -> None:
    """h[:rows] += sum over ranks of slots[:, :rows]; x = rmsnorm(h) * w."""
    world, _, cols = slots.shape
    _rt.launch(_IMG, "fb_add_rmsnorm_slots", (rows,), (256,), [
        slots.data_ptr(), world, slots.stride(0), h.data_ptr(), w.data_ptr(), x.data_ptr(), rows, cols, float(eps)])


def argmax_sharded(symm: SymmetricMemory, logits: torch.Tensor, vocab_offset: int, pairs_offset: int,
                   out: torch.Tensor) -> None:
    """Greedy token over a vocab-sharded lm_head: local shard argmax -> (value,
    index) pairs exchanged -> barrier -> the same global argmax on every rank."""
    t, v = logits.shape
    s = symm
    _rt.launch(_IMG, "fb_argmax_shard", (t,), (512,), [
        logits.data_ptr(), logits.stride(0), t, v, vocab_offset, s.mc_ptr if s.multicast else 0, s.base, s.stride,
        pairs_offset, s.rank, s.world])
    barrier(s)
    pairs = s.tensor(s.rank, (s.world, t, 2), torch.int32, pairs_offset)
    _rt.launch(_IMG, "fb_argmax_combine", (math.ceil(t / 128),), (128,), [pairs.data_ptr(), t, s.world, out.data_ptr()])


__all__ = ["CTRL_BYTES", "SlotExchange", "add_rmsnorm_slots", "all_reduce", "argmax_sharded", "barrier"]
