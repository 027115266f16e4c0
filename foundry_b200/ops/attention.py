"""Attention ops (csrc/kernels/attention.cu): paged split-KV decode attention
and causal prefill attention. head_dim is 128 and the KV page is 64 tokens."""

from __future__ import annotations

import math

import torch

from . import _rt

_IMG = "attention"
PAGE = 64
LOG2E = 1.4426950408889634


def decode_smem(group: int) -> int:
    return 2 * 2 * PAGE * 128 * 2 + (group * PAGE * 2 + group + group * 128) * 4


def decode_splits(batch: int, n_kv: int, max_pages: int, sms: int | None = None) -> tuple[int, int]:
    """(num_splits, pages_per_split) so that batch * n_kv * splits work items
    fill the GPU. pages_per_split is even: the tensor-core kernel works in
    128-token (two-page) chunks."""
    sms = sms or _rt.sm_count()
    max_chunks = math.ceil(max_pages / 2)
    want = max(1, math.ceil(2 * sms / max(1, batch * n_kv)))
    splits = max(1, min(want, max_chunks))
    cps = math.ceil(max_chunks / splits)
    splits = math.ceil(max_chunks / cps)
    return splits, 2 * cps


_tmaps: dict[tuple, bytes] = {}


def _cache_tmap(cache: torch.Tensor, box_rows: int = 64) -> bytes:
    """TMA map of a paged cache [blocks, Hkv, 64, 128] viewed as [rows, 128]:
    64-column x ``box_rows`` boxes, 128B swizzle (64 rows load whole pages, 16
    rows the live row blocks of a sequence's last page)."""
    key = (cache.data_ptr(), cache.shape, box_rows)
    m = _tmaps.get(key)
    if m is None:
        from .._native import core

        rows = cache.shape[0] * cache.shape[1] * cache.shape[2]
        m = core().make_tmap_2d(cache.data_ptr(), 9, 128, rows, 256, 64, box_rows, 3)
        if len(_tmaps) > 4096:
            _tmaps.clear()
        _tmaps[key] = m
    return m


# Dynamic shared memory of the tensor-core kernel by ring depth (1 stage: three CTAs per SM).
TC_SMEM = {3: 208 * 1024, 1: 74 * 1024}


class DecodeWorkspace:
    def __init__(self, max_batch: int, n_q: int, max_splits: int, device=None,
                 o_part: torch.Tensor | None = None, ml_part: torch.Tensor | None = None):
        device = device or torch.device("cuda", torch.cuda.current_device())
        n = max_batch * n_q * max_splits
        self.o_part = o_part if o_part is not None else torch.empty(n * 128, dtype=torch.float32, device=device)
        self.ml_part = ml_part if ml_part is not None else torch.empty(n * 2, dtype=torch.float32, device=device)
        self.capacity = n


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_tables: torch.Tensor,
                     seq_lens: torch.Tensor, out: torch.Tensor, max_pages: int, ws: DecodeWorkspace,
                     scale: float | None = None, splits: tuple[int, int] | None = None,
                     impl: str = "tc") -> torch.Tensor:
    """q: [B, Hq, 128]; caches [blocks, Hkv, 64, 128]; block_tables [B, max_blocks] int32;
    seq_lens [B] int32 (tokens in cache incl. the current one). The launch
    covers ``max_pages`` pages per sequence so its shape is static.

    ``impl="tc"``: tcgen05 kernel (csrc/kernels/attention_tc.cu, persistent
    grid); ``impl="simt"``: CUDA-core flash-decoding kernel (attention.cu)."""
    b, n_q, d = q.shape
    assert d == 128 and k_cache.shape[2] == PAGE
    n_kv = k_cache.shape[1]
    g = n_q // n_kv
    if g not in (4, 8):
        raise ValueError(f"GQA group {g} not supported (4 or 8)")
    scale = scale if scale is not None else 1.0 / math.sqrt(d)
    s, pps = splits or decode_splits(b, n_kv, max_pages)
    if s > 1 and b * n_q * s > ws.capacity:
        raise RuntimeError("decode attention workspace too small")
    if impl in ("tc", "tc1", "tc3"):
        if pps % 2:
            raise ValueError("pages_per_split must be even for the tensor-core kernel")
        stages = 3 if impl == "tc3" else 1
        ctas_per_sm = 3 if stages == 1 else 1
        items = b * n_kv * s
        grid = min(items, _rt.sm_count() * ctas_per_sm)
        _rt.launch("attention_tc", f"fb_decode_attn_tc_g{g}_s{stages}", (grid,), (192,), [
            _cache_tmap(k_cache), _cache_tmap(v_cache), _cache_tmap(k_cache, 16), _cache_tmap(v_cache, 16),
            q.data_ptr(), block_tables.data_ptr(),
            block_tables.shape[1], seq_lens.data_ptr(), out.data_ptr(), ws.o_part.data_ptr(), ws.ml_part.data_ptr(),
            b, n_kv, s, pps // 2, float(scale * LOG2E),
        ], smem=TC_SMEM[stages])
    else:
        _rt.launch(_IMG, f"fb_decode_attn_g{g}", (s, n_kv, b), (128,), [
            q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), block_tables.data_ptr(), block_tables.shape[1],
            seq_lens.data_ptr(), out.data_ptr(), ws.o_part.data_ptr(), ws.ml_part.data_ptr(), n_kv, pps,
            float(scale * LOG2E),
        ], smem=decode_smem(g))
    if s > 1:
        _rt.launch(_IMG, "fb_decode_attn_combine", (b, n_q), (128,), [
            ws.o_part.data_ptr(), ws.ml_part.data_ptr(), out.data_ptr(), n_q, s,
        ])
    return out


PREFILL_TILE = {"tc": 128, "simt": 64}
PREFILL_TC_SMEM = 200 * 1024


def prefill_tiles(seqlens: list[int], tile: int = 128) -> tuple[list[int], list[int]]:
    """(sequence, first query position) of every ``tile``-row query tile."""
    tile_seq, tile_start = [], []
    for i, n in enumerate(seqlens):
        for s0 in range(0, n, tile):
            tile_seq.append(i)
            tile_start.append(s0)
    return tile_seq, tile_start


def _rows_tmap(t: torch.Tensor) -> bytes:
    """TMA map of a [T, heads * 128] bf16 view: 64-dim x 128-row boxes, 128B swizzle."""
    from .._native import core

    rows, cols = t.shape
    if t.stride(1) != 1 or (t.stride(0) * 2) % 16 or t.data_ptr() % 16:
        raise ValueError("prefill q/k/v must be row-contiguous with 16-byte aligned rows")
    return core().make_tmap_2d(t.data_ptr(), 9, cols, rows, t.stride(0) * 2, 64, 128, 3)


def prefill_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor,
                      cu_seqlens: torch.Tensor, tile_seq: torch.Tensor, tile_start: torch.Tensor,
                      n_q: int, n_kv: int, scale: float | None = None, impl: str = "tc") -> torch.Tensor:
    """Causal attention over packed prompts. q: [T, *] with head h at columns
    h*128 (row stride q.stride(0)); k, v likewise with n_kv heads; out [T, n_q*128].

    ``impl="tc"``: tcgen05 kernel (csrc/kernels/prefill_tc.cu), query tiles of
    128 rows; ``impl="simt"``: CUDA-core kernel, query tiles of 64 rows. The
    tile tables must come from ``prefill_tiles(seqlens, PREFILL_TILE[impl])``."""
    scale = scale if scale is not None else 1.0 / math.sqrt(128)
    n_tiles = tile_seq.numel()
    if impl == "tc":
        t = q.shape[0]
        _rt.launch("prefill_tc", "fb_prefill_attn_tc", (n_tiles, n_q), (192,), [
            _rows_tmap(q[:t, : n_q * 128]), _rows_tmap(k[:t, : n_kv * 128]), _rows_tmap(v[:t, : n_kv * 128]),
            out.data_ptr(), out.stride(0), cu_seqlens.data_ptr(), tile_seq.data_ptr(), tile_start.data_ptr(), n_q,
            n_kv, float(scale * LOG2E)], smem=PREFILL_TC_SMEM)
        return out
    _rt.launch(_IMG, "fb_prefill_attn", (n_tiles, n_q), (128,), [
        q.data_ptr(), k.data_ptr(), v.data_ptr(), q.stride(0), k.stride(0), v.stride(0), out.data_ptr(),
        out.stride(0),
        cu_seqlens.data_ptr(), tile_seq.data_ptr(), tile_start.data_ptr(), n_q, n_kv, float(scale * LOG2E),
    ])
    return out
