"""Memory-bound ops (csrc/kernels/elementwise.cu): init, embedding, RMSNorm,
SiLU*mul, (QK-norm +) RoPE + paged KV write, argmax, decode bookkeeping."""

from __future__ import annotations

import math

import torch

from . import _rt
from .gemm import Partial

_IMG = "elementwise"


def _grid_1d(n: int, per_block: int, cap: int = 148 * 16) -> int:
    return max(1, min(math.ceil(n / per_block), cap))


def init_normal_(t: torch.Tensor, seed: int, std: float = 0.02, mean: float = 0.0) -> torch.Tensor:
    """Deterministic N(mean, std) fill of a bf16 tensor: element i depends only
    on (seed, i), so two processes produce identical weights."""
    assert t.dtype == torch.bfloat16 and t.is_contiguous()
    n = t.numel()
    _rt.launch(_IMG, "fb_init_normal_bf16", (_grid_1d(n // 2 + 1, 256),), (256,),
               [t.data_ptr(), n, seed & ((1 << 64) - 1), float(mean), float(std)])
    return t


def fill_(t: torch.Tensor, value: float) -> torch.Tensor:
    assert t.dtype == torch.bfloat16 and t.is_contiguous()
    _rt.launch(_IMG, "fb_fill_bf16", (_grid_1d(t.numel(), 256),), (256,), [t.data_ptr(), t.numel(), float(value)])
    return t


def embedding(ids: torch.Tensor, table: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    t_tok = ids.numel()
    vocab, h = table.shape
    assert h % 8 == 0 and ids.dtype == torch.int32
    _rt.launch(_IMG, "fb_embedding", (t_tok,), (128,), [ids.data_ptr(), table.data_ptr(), out.data_ptr(), t_tok, h, vocab])
    return out


def rmsnorm(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor, eps: float) -> torch.Tensor:
    t_tok, h = x.shape
    assert h % 8 == 0 and x.is_contiguous() and out.is_contiguous()
    _rt.launch(_IMG, "fb_rmsnorm", (t_tok,), (256,), [x.data_ptr(), w.data_ptr(), out.data_ptr(), t_tok, h, float(eps)])
    return out


def silu_mul(gu: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    t_tok, two_i = gu.shape
    i = two_i // 2
    assert i % 8 == 0
    _rt.launch(_IMG, "fb_silu_mul", (_grid_1d(t_tok * i // 8, 256),), (256,), [gu.data_ptr(), out.data_ptr(), t_tok, i])
    return out


def rope_cos_sin(max_pos: int, theta: float, head_dim: int = 128, device=None,
                 scaling: dict | None = None) -> torch.Tensor:
    """fp32 (cos, sin) table [max_pos, head_dim/2, 2] for half-rotation RoPE.

    ``scaling`` supports the Llama-3.1 frequency remap
    (rope_type="llama3": factor, low_freq_factor, high_freq_factor,
    original_max_position_embeddings).
    """
    half = head_dim // 2
    inv = 1.0 / (theta ** (torch.arange(0, half, dtype=torch.float64) * 2 / head_dim))
    if scaling and scaling.get("rope_type") == "llama3":
        factor = scaling["factor"]
        lo, hi = scaling["low_freq_factor"], scaling["high_freq_factor"]
        old = scaling["original_max_position_embeddings"]
        wavelen = 2 * math.pi / inv
        smooth = (old / wavelen - lo) / (hi - lo)
        scaled = torch.where(wavelen > old / lo, inv / factor, inv)
        mid = (wavelen <= old / lo) & (wavelen >= old / hi)
        inv = torch.where(mid, (1 - smooth) * inv / factor + smooth * inv, scaled)
    pos = torch.arange(max_pos, dtype=torch.float64)
    ang = torch.outer(pos, inv)
    return torch.stack([ang.cos(), ang.sin()], dim=-1).to(torch.float32).contiguous().to(device)


def rope_kv_write(qkv, positions: torch.Tensor, cos_sin: torch.Tensor, q_out: torch.Tensor,
                  k_cache: torch.Tensor, v_cache: torch.Tensor, slots: torch.Tensor, n_q: int, n_kv: int,
                  q_norm: torch.Tensor | None = None, k_norm: torch.Tensor | None = None,
                  eps: float = 1e-6, k_out: torch.Tensor | None = None, v_out: torch.Tensor | None = None) -> None:
    """Rotates q (into q_out [T, n_q, 128]) and k, writes k/v into the paged
    caches [blocks, n_kv, page, 128]; optional per-head RMSNorm on q/k first.
    ``qkv`` is the bf16 [T, (n_q+2n_kv)*128] GEMM output or a ``Partial``
    (split-K slices, summed here). With ``k_out``/``v_out`` the rotated k and
    the v heads are also written packed [T, n_kv, 128]."""
    if isinstance(qkv, Partial):
        t_tok, ld = qkv.rows, qkv.cols
        src, part, s, stride = 0, qkv.buf.data_ptr(), qkv.splits, qkv.stride
    else:
        t_tok, ld = qkv.shape[0], qkv.stride(0)
        src, part, s, stride = qkv.data_ptr(), 0, 0, 0
    page = k_cache.shape[2]
    use_norm = 1 if q_norm is not None else 0
    heads = n_q + 2 * n_kv
    _rt.launch(_IMG, "fb_rope_kv_write", (t_tok, math.ceil(heads / 8)), (256,), [
        src, ld, positions.data_ptr(), cos_sin.data_ptr(),
        q_norm.data_ptr() if use_norm else 0, k_norm.data_ptr() if use_norm else 0, float(eps), use_norm,
        q_out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), slots.data_ptr(), t_tok, n_q, n_kv, page,
        k_out.data_ptr() if k_out is not None else 0, v_out.data_ptr() if v_out is not None else 0,
        part, s, stride,
    ])


def add_rmsnorm_partials(p: Partial, h: torch.Tensor, w: torch.Tensor, x: torch.Tensor, eps: float) -> None:
    """h = bf16(sum of split slices + h); x = rmsnorm(h) * w (one pass)."""
    t_tok, hid = h.shape
    assert p.rows == t_tok and p.cols == hid and h.is_contiguous() and x.is_contiguous()
    _rt.launch(_IMG, "fb_add_rmsnorm_partials", (t_tok,), (256,), [
        p.buf.data_ptr(), p.splits, p.stride, h.data_ptr(), w.data_ptr(), x.data_ptr(), t_tok, hid, float(eps)])


def argmax(logits: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    t_tok, v = logits.shape
    _rt.launch(_IMG, "fb_argmax", (t_tok,), (512,), [logits.data_ptr(), out.data_ptr(), t_tok, v, logits.stride(0)])
    return out


def decode_advance(seq_lens: torch.Tensor, positions: torch.Tensor, slots: torch.Tensor,
                   block_tables: torch.Tensor, page: int, active: torch.Tensor | None = None) -> None:
    b = seq_lens.numel()
    _rt.launch(_IMG, "fb_decode_advance", (math.ceil(b / 128),), (128,), [
        seq_lens.data_ptr(), positions.data_ptr(), slots.data_ptr(), block_tables.data_ptr(),
        block_tables.shape[1], page, b, active.data_ptr() if active is not None else 0,
    ])


def copy_i32(src: torch.Tensor, dst: torch.Tensor) -> None:
    n = src.numel()
    _rt.launch(_IMG, "fb_copy_i32", (math.ceil(n / 256),), (256,), [src.data_ptr(), dst.data_ptr(), n])
