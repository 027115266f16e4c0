"""Block-scaled fp8 linear layers and mixture-of-experts ops
(csrc/kernels/moe.cu).

Format: weights are e4m3 with one fp32 scale per 128 x 128 block, activations
e4m3 with one fp32 scale per token per 128 features (the "fp8 block" format
of the Qwen3/DeepSeek fp8 checkpoints the reference serves through vLLM /
SGLang with DeepGEMM, reference recipe/sglang/serve_qwen3-30ba3bfp8_ep.sh:51-70).

The grouped GEMM works from a device-side chunk table ({expert, first row,
rows}), so one static launch serves any expert load - the property that
makes MoE decode capturable in a CUDA graph. A dense fp8 linear layer is the
same kernel with one expert and a chunk table over the token rows.

Decode flow of one MoE block (single GPU):
    router logits (bf16 GEMM) -> topk -> plan (counts, sorted positions,
    chunks) -> dispatch_local (quantise + scatter) -> grouped GEMM gate_up
    -> silu_mul_quant -> grouped GEMM down -> combine_add_rmsnorm
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from .._native import core
from . import _rt

_IMG = "moe"
QBLK = 128
_U8 = 0  # CU_TENSOR_MAP_DATA_TYPE_UINT8
_SWIZZLE_128B = 3
MAX_KB = 32
EPI_RESIDUAL = 2
EPI_W_STREAM = 4
EPI_PEER_COMBINE = 32
NBUF = 8


# resident CTAs per SM of the promote GEMM per token-tile width (MoeOcc in
# moe.cu): one CTA's per-k-block promotion chain, not HBM, bounds 32-token tiles
GEMM_CTAS = {32: 3, 64: 1}


def gemm_smem(bn: int) -> int:
    stage = 128 * QBLK + bn * QBLK
    budget = {1: 200, 2: 100, 3: 60}[GEMM_CTAS[bn]] * 1024
    stages = min(10, budget // stage)
    return stages * stage + 3 * bn * MAX_KB * 4 + 2 * MAX_KB * 4 + 8 * (2 * stages + 2 * NBUF + 4) + 16 + 1024


def kb_pad(kb: int) -> int:
    """Scale rows are padded to a multiple of 4 floats (16-byte rows for bulk copies)."""
    return (kb + 3) // 4 * 4


def scale_rows(rows: int) -> int:
    """Rows of an activation-scale buffer for ``rows`` tokens: the GEMM
    fetches a whole chunk of up to 64 rows of scales at once."""
    return rows + 64


def act_buffers(arena, rows: int, k: int):
    """(e4m3 [rows, k], fp32 scales [rows + 64, kb_pad(k / 128)]) zeroed activation buffers."""
    q = arena.zeros((rows, k), torch.uint8)
    s = arena.zeros((scale_rows(rows), kb_pad(k // QBLK)), torch.float32)
    return q, s


@dataclass
class Fp8Weight:
    """e4m3 weight ``q`` viewed as [experts * rows, cols] (uint8) with fp32
    block scales ``scale`` [experts, rows / 128, kb_pad(cols / 128)] (the
    padding columns are unused)."""

    q: torch.Tensor
    scale: torch.Tensor
    experts: int
    rows: int  # output features per expert
    cols: int  # input features

    @staticmethod
    def empty(arena, experts: int, rows: int, cols: int) -> "Fp8Weight":
        if rows % 128 or cols % 128:
            raise ValueError(f"fp8 block weights need multiples of 128, got {rows} x {cols}")
        q = arena.empty((experts * rows, cols), torch.uint8)
        s = arena.zeros((experts, rows // 128, kb_pad(cols // 128)), torch.float32)
        return Fp8Weight(q, s, experts, rows, cols)

    def dequant(self) -> torch.Tensor:
        """fp32 [experts * rows, cols] (tests, reference forward)."""
        w = self.q.view(torch.float8_e4m3fn).float().view(self.experts, self.rows // 128, 128, self.cols // 128, 128)
        sc = self.scale[:, :, : self.cols // 128]
        return (w * sc[:, :, None, :, None]).reshape(self.experts * self.rows, self.cols)


_tmaps: dict[tuple, bytes] = {}


def fp8_tmap(t: torch.Tensor, box_rows: int) -> bytes:
    """TMA map of a row-major [rows, K] e4m3 (uint8) matrix, 128-byte x box_rows boxes, 128B swizzle."""
    rows, k = t.shape
    key = (t.data_ptr(), rows, k, box_rows)
    m = _tmaps.get(key)
    if m is None:
        if t.stride(1) != 1 or t.stride(0) != k or k % 16 or t.data_ptr() % 16:
            raise ValueError("fp8 GEMM operands must be contiguous with 16-byte aligned rows")
        m = core().make_tmap_2d(t.data_ptr(), _U8, k, rows, k, QBLK, box_rows, _SWIZZLE_128B)
        if len(_tmaps) > 8192:
            _tmaps.clear()
        _tmaps[key] = m
    return m


def init_fp8_block_(w: Fp8Weight, seed: int, std: float, row_offset: int = 0) -> None:
    """Random N(0, std) weights quantised per 128 x 128 block, generated in
    place. Row r draws the values of row r + row_offset of the full matrix,
    so a shard of experts matches the unsharded weights."""
    r, c = w.experts * w.rows, w.cols
    _rt.launch(_IMG, "fb_init_fp8_block", (c // 128, r // 128), (256,),
               [w.q.data_ptr(), w.scale.data_ptr(), r, c, seed & ((1 << 64) - 1), float(std), int(row_offset)])


def quantize_block_fp8_(w_bf16: torch.Tensor, w: Fp8Weight) -> None:
    """Quantises a bf16 [experts * rows, cols] matrix into ``w``."""
    r, c = w_bf16.shape
    assert (r, c) == tuple(w.q.shape) and w_bf16.is_contiguous()
    _rt.launch(_IMG, "fb_quant_block_fp8", (c // 128, r // 128), (256,),
               [w_bf16.data_ptr(), r, c, w.q.data_ptr(), w.scale.data_ptr()])


def dequantize_block_fp8_(w: Fp8Weight, out: torch.Tensor) -> torch.Tensor:
    """bf16 [experts * rows, cols] <- e4m3 * block scale (one rounding to bf16)."""
    r, c = w.experts * w.rows, w.cols
    assert tuple(out.shape) == (r, c) and out.dtype == torch.bfloat16 and out.is_contiguous()
    _rt.launch(_IMG, "fb_dequant_block_fp8", (c // 128, r // 128), (256,),
               [w.q.data_ptr(), w.scale.data_ptr(), r, c, out.data_ptr()])
    return out


def quantize_rows(x: torch.Tensor, xq: torch.Tensor, xs: torch.Tensor, pos: torch.Tensor | None = None,
                  topk: int = 1) -> None:
    """x [T, H] bf16 -> e4m3 rows with per-128 scales (``xs`` rows padded to
    kb_pad(H / 128) floats). With ``pos`` ([T, topk] int32) row t is written
    to rows pos[t, :] (MoE dispatch); else to row t."""
    t, h = x.shape
    if h % QBLK:
        raise ValueError(f"hidden {h} must be a multiple of 128")
    warps = t * math.ceil(h // QBLK / 4)
    _rt.launch(_IMG, "fb_moe_dispatch_local", (math.ceil(warps / 8),), (256,), [
        x.data_ptr(), x.stride(0), t, h, pos.data_ptr() if pos is not None else 0, topk, xq.data_ptr(),
        xs.data_ptr()])


def dense_chunks(t: int, bn: int, chunks: torch.Tensor, meta: torch.Tensor) -> None:
    _rt.launch(_IMG, "fb_moe_dense_chunks", (1,), (256,), [t, bn, chunks.data_ptr(), meta.data_ptr()])


def gemm_fp8(w: Fp8Weight, xq: torch.Tensor, xs: torch.Tensor, chunks: torch.Tensor, meta: torch.Tensor,
             out: torch.Tensor | int, max_units: int, bn: int = 64, residual: torch.Tensor | None = None,
             stream_weights: bool = False, prefetch: int = 0, peer_rowmap: torch.Tensor | None = None,
             peer_stride: int = 0, ldo: int | None = None) -> torch.Tensor | int:
    """Grouped (or, with one expert, dense) block-scaled fp8 GEMM:
    out[r, :rows] = dequant(W[expert(r)]) @ dequant(xq[r]) for every row r of
    every chunk in the table (+ residual). ``max_units`` bounds the chunks x
    row-blocks of any step and sizes the persistent grid. ``stream_weights``
    hints weight tiles evict-first in L2 (experts whose tiles are read once).

    Expert-parallel combine: with ``peer_rowmap`` (int32 per output row:
    source rank << 24 | row) ``out`` is the address of the combine buffer in
    rank 0's symmetric window and each row is stored over NVLink into rank
    ``map >> 24``'s window (``peer_stride`` bytes apart), row ``map & 0xFFFFFF``."""
    if bn not in (32, 64):
        raise ValueError("bn must be 32 or 64")
    if w.cols // QBLK > MAX_KB:
        raise ValueError(f"K = {w.cols} exceeds {MAX_KB * QBLK}")
    mode = 0
    if residual is not None:
        assert residual.stride() == out.stride()
        mode |= EPI_RESIDUAL
    if stream_weights:
        mode |= EPI_W_STREAM
    mode |= (min(prefetch, 15) & 15) << 12
    if peer_rowmap is not None:
        mode |= EPI_PEER_COMBINE
        out_ptr, res_ptr, ld = int(out), peer_rowmap.data_ptr(), int(ldo)
    else:
        out_ptr, res_ptr, ld = out.data_ptr(), residual.data_ptr() if residual is not None else 0, out.stride(0)
    grid = max(1, min(max_units, GEMM_CTAS[bn] * _rt.sm_count()))
    _rt.launch(_IMG, f"fb_moe_gemm_fp8_bn{bn}", (grid,), (192,), [
        fp8_tmap(w.q, 128), fp8_tmap(xq, bn), w.scale.data_ptr(), xs.data_ptr(), chunks.data_ptr(),
        meta.data_ptr(), out_ptr, res_ptr, w.rows, w.cols, ld, mode, int(peer_stride)], smem=gemm_smem(bn))
    return out


def w8_smem(bn: int) -> int:
    stage = 128 * 128 + bn * 128 * 2
    cbuf = 2 * 128 * 128 * 2
    stages = min(6, (216 * 1024 - cbuf) // stage)
    return 1024 + cbuf + stages * stage + 2 * MAX_KB * 4 + 8 * (2 * stages + 2 * 2 + 8) + 16


def gemm_w8(w: Fp8Weight, x: torch.Tensor, chunks: torch.Tensor, meta: torch.Tensor, out: torch.Tensor,
            max_units: int, bn: int = 64, residual: torch.Tensor | None = None,
            stream_weights: bool = False, prefetch: int = 0) -> torch.Tensor:
    """Weight-only fp8 grouped / dense GEMM: out[r, :rows] = dequant(W[expert(r)]) @ x[r]
    for every row r of every chunk in the table (+ residual), x in bf16. The
    e4m3 weight tiles are dequantised on chip into bf16 and multiplied on the
    tcgen05 bf16 path with the whole K loop accumulated in TMEM."""
    from .gemm import tmap as bf16_tmap

    if bn not in (32, 64, 128):
        raise ValueError("bn must be 32, 64 or 128")
    if w.cols // QBLK > MAX_KB or x.shape[1] != w.cols:
        raise ValueError(f"bad K: weights {w.cols}, activations {x.shape[1]}")
    mode = 0
    if residual is not None:
        assert residual.stride() == out.stride()
        mode |= EPI_RESIDUAL
    if stream_weights:
        mode |= EPI_W_STREAM
    mode |= (min(prefetch, 15) & 15) << 12
    grid = max(1, min(max_units, _rt.sm_count()))
    _rt.launch(_IMG, f"fb_moe_gemm_w8_bn{bn}", (grid,), (320,), [
        fp8_tmap(w.q, 128), bf16_tmap(x, bn), w.scale.data_ptr(), chunks.data_ptr(), meta.data_ptr(),
        out.data_ptr(), residual.data_ptr() if residual is not None else 0, w.rows, w.cols, out.stride(0), mode],
        smem=w8_smem(bn))
    return out


def scatter_rows(x: torch.Tensor, pos: torch.Tensor, topk: int, dst: torch.Tensor) -> None:
    """dst[pos[t, j]] = x[t] for every token t and slot j (expert-sorted gather, bf16)."""
    t, h = x.shape
    _rt.launch(_IMG, "fb_moe_scatter_rows", (t,), (256,), [x.data_ptr(), x.stride(0), t, h, pos.data_ptr(), topk,
                                                          dst.data_ptr()])


def topk(logits: torch.Tensor, k: int, ids: torch.Tensor, weights: torch.Tensor, renorm: bool = True) -> None:
    t, e = logits.shape
    if e % 32 or e > 256 or k > 8:
        raise ValueError("experts must be a multiple of 32 and <= 256, top-k <= 8")
    _rt.launch(_IMG, "fb_moe_topk", (math.ceil(t / 8),), (256,), [
        logits.data_ptr(), logits.stride(0), t, e, k, 1 if renorm else 0, ids.data_ptr(), weights.data_ptr()])


def plan(ids: torch.Tensor, pairs: int, experts: int, bn: int, pos: torch.Tensor, counts: torch.Tensor,
         chunks: torch.Tensor, meta: torch.Tensor) -> None:
    """Per-expert counts, stable expert-sorted positions of the ``pairs``
    (token, slot) pairs in ``ids`` and the chunk table (<= bn rows each)."""
    _rt.launch(_IMG, "fb_moe_plan", (1,), (1024,), [
        ids.data_ptr(), pairs, experts, bn, pos.data_ptr(), counts.data_ptr(), chunks.data_ptr(), meta.data_ptr()])


def max_chunks(pairs: int, experts: int, bn: int) -> int:
    return pairs // bn + experts


def silu_mul_quant(gu: torch.Tensor, rows: int, aq: torch.Tensor, as_: torch.Tensor,
                   meta: torch.Tensor | None = None) -> None:
    """gu [rows, 2I] (gate | up) -> e4m3 silu(gate) * up [rows, I] + per-128 scales."""
    i = gu.shape[1] // 2
    _rt.launch(_IMG, "fb_moe_silu_mul_quant", (math.ceil(rows / 8),), (256,), [
        gu.data_ptr(), rows, i, meta.data_ptr() if meta is not None else 0, aq.data_ptr(), as_.data_ptr()])


def combine_add_rmsnorm(y: torch.Tensor, pos: torch.Tensor, weights: torch.Tensor, k: int, h: torch.Tensor,
                        norm_w: torch.Tensor, x: torch.Tensor, eps: float) -> None:
    """h[t] += sum_j weights[t, j] * y[pos[t, j]]; x = rmsnorm(h) * norm_w."""
    t, hd = h.shape
    if hd % 8 or hd > 4096:
        raise ValueError("hidden must be a multiple of 8 and <= 4096")
    _rt.launch(_IMG, "fb_moe_combine_add_rmsnorm", (t,), (256,), [
        y.data_ptr(), y.stride(0), pos.data_ptr(), weights.data_ptr(), k, h.data_ptr(), norm_w.data_ptr(),
        x.data_ptr(), t, hd, float(eps)])


__all__ = [
    "Fp8Weight", "combine_add_rmsnorm", "dense_chunks", "fp8_tmap", "gemm_fp8", "gemm_smem", "gemm_w8", "init_fp8_block_",
    "scatter_rows", "w8_smem", "dequantize_block_fp8_",
    "max_chunks", "plan", "quantize_block_fp8_", "quantize_rows", "silu_mul_quant", "topk",
]
