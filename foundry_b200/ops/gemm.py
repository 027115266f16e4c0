"""bf16 linear layers on the tcgen05 GEMM (csrc/kernels/gemm_bf16.cu).

``linear(x, w)`` computes ``x @ w.T`` (nn.Linear layout: ``w`` is
[out_features, in_features]). Small token counts (decode) run "swap-AB": the
weight rows fill the 128-row MMA M dimension and the tokens become the MMA N
dimension (16..256); the output is written transposed back to [tokens, out].

When a problem has too few output tiles to occupy every SM, the planner
splits K. Split GEMMs do not reduce in-kernel: each split writes its fp32
slice of the output and ``linear`` returns a ``Partial`` that the consuming
op (``add_rmsnorm_partials``, ``rope_kv_write``, ``reduce_partials``) sums
while it reads its input. Callers that cannot consume slices pass no
``partials`` buffer and get an unsplit GEMM.
"""

from __future__ import annotations

import functools
import math
import os
from dataclasses import dataclass

import torch

from .._native import core
from . import _rt

BM, BK = 128, 64
EPI_TRANSPOSE, EPI_RESIDUAL, EPI_A_STREAM, EPI_B_STREAM = 1, 2, 4, 8
EPI_MCAST = 1 << 16
EPI_TMA_OUT = 1 << 17
EPI_A_CONST = 1 << 18  # A (the weights of a swap-AB GEMM) may be loaded before the PDL wait
EPI_SWIGLU = 1 << 19  # two A tiles per unit (gate rows, up rows); the epilogue writes silu(gate) * up
EPI_COLS = 32  # tokens per epilogue store chunk of the one-SM kernel
_BF16 = 9  # CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
_F32 = 7  # CU_TENSOR_MAP_DATA_TYPE_FLOAT32
_NO_MAP = bytes(128)  # placeholder for tensor-map parameters a launch does not use
_SWIZZLE_128B = 3
_BNS = (16, 32, 64, 128, 256)
# Cost model constants (measured on B200): per-CTA shared-memory fill rate of
# the TMA pipeline, per-SM bf16 tensor rate, and achievable HBM bandwidth.
_CTA_FILL_BPS = 90e9
_CTA_FILL_BPS_MAX = 150e9
_TMA_LATENCY = 2.0e-6
_SM_MMA_FLOPS = 14e12
_HBM_BPS = 6.0e12
MAX_SPLITS = 8


STG_BYTES = 64 * BM * 4  # fp32 staging of the transposed epilogue (csrc/kernels/gemm_bf16.cu)


def smem_bytes(bn: int, mt: int = 1) -> int:
    """Dynamic shared memory of the one-SM kernels (and the stream-K ones,
    which use the same ring): ring of 192 KB at most, staging, barriers."""
    stage = mt * BM * BK * 2 + bn * BK * 2
    stages = min(8, (192 * 1024) // stage)
    return stages * stage + STG_BYTES + 1024 + 256


def smem_bytes_pair(bn: int) -> int:
    """Shared memory of one CTA of the two-SM kernel (its 128 A rows + bn/2 B
    rows per stage, ring of 192 KB at most), staging, barriers."""
    stage = BM * BK * 2 + (bn // 2) * BK * 2
    stages = min(8, (192 * 1024) // stage)
    return stages * stage + STG_BYTES + 1024 + 256


# Two-SM (cta_group::2) tiles for swap-AB decode GEMMs: "auto" (default) uses
# them, with 256-token tiles, for 256-token batches; "1" for every swap plan
# with tiles of 64+ tokens; "0" never. Measured on B200 at 256 tokens with both
# kernels on the staged TMA-store epilogue (CUDA graph of 20 launches, L2
# flushed before each, programmatic dependent launch; us, one-SM -> two-SM):
# qkv 19.8 -> 19.3, o 17.5 -> 16.6 (4 splits), down 36.7 -> 31.9, lm_head
# 242.5 -> 225.3. Each SM loads half the token tile per k-block, so a stage
# is 32 KB instead of 48 KB at the same tensor work.
_PAIR = os.environ.get("FOUNDRY_GEMM_PAIR", "auto")


@dataclass
class Partial:
    """fp32 split-K slices of a GEMM output: ``buf[s * stride + row * cols + col]``."""

    buf: torch.Tensor
    splits: int
    rows: int
    cols: int

    @property
    def stride(self) -> int:
        return self.rows * self.cols


class StreamKBuffer:
    """Workspace of the stream-K GEMM: fp32 partial tiles (``ws``, any
    contents; may share memory with a PartialBuffer whose slices are consumed
    before and produced after the stream-K GEMM) and ``flags`` (int32, must be
    zero before the first launch; every launch leaves them zero)."""

    def __init__(self, ws: torch.Tensor, flags: torch.Tensor):
        assert ws.dtype == torch.float32 and flags.dtype == torch.int32
        self.ws, self.flags = ws, flags

    def fits(self, grid: int, bn: int) -> bool:
        return self.ws.numel() >= grid * BM * bn and self.flags.numel() >= grid * 8


class PartialBuffer:
    """Scratch for split slices (fp32). Must not be shared by GEMMs whose
    slices are still unconsumed."""

    def __init__(self, numel: int | None = None, device=None, buf: torch.Tensor | None = None):
        device = device or torch.device("cuda", torch.cuda.current_device())
        self.buf = buf if buf is not None else torch.empty(numel, dtype=torch.float32, device=device)

    @property
    def numel(self) -> int:
        return self.buf.numel()


_tmaps: dict[tuple, bytes] = {}


def tmap(t: torch.Tensor, box_rows: int) -> bytes:
    """TMA descriptor of a row-major [rows, K] bf16 matrix, 64 x box_rows boxes, 128B swizzle."""
    rows, k = t.shape
    ld = t.stride(0)
    key = (t.data_ptr(), rows, k, ld, box_rows)
    m = _tmaps.get(key)
    if m is None:
        if t.stride(1) != 1 or (ld * 2) % 16 or t.data_ptr() % 16:
            raise ValueError("GEMM operands must be K-contiguous with 16-byte aligned rows")
        m = core().make_tmap_2d(t.data_ptr(), _BF16, k, rows, ld * 2, BK, box_rows, _SWIZZLE_128B)
        if len(_tmaps) > 8192:
            _tmaps.clear()
        _tmaps[key] = m
    return m


_omaps: dict[tuple, bytes] = {}


def _cached_map(key: tuple, make) -> bytes:
    m = _omaps.get(key)
    if m is None:
        m = make()
        if len(_omaps) > 8192:
            _omaps.clear()
        _omaps[key] = m
    return m


def out_maps(out_ptr: int, res_ptr: int, n_out: int, t_tok: int, ldo: int, bn: int) -> tuple[bytes, bytes] | None:
    """TMA-store maps of a transposed bf16 output [t_tok, ldo] (and of its
    residual), 128 features x min(bn, 32) tokens per box; None when the rows
    are not 16-byte aligned (the kernel then stores element by element)."""
    if (ldo * 2) % 16 or out_ptr % 16 or (res_ptr and res_ptr % 16):
        return None
    rows = min(bn, EPI_COLS)

    def make(ptr):
        return lambda: core().make_tmap_2d(ptr, _BF16, n_out, t_tok, ldo * 2, BM, rows, 0)

    o = _cached_map(("o", out_ptr, n_out, t_tok, ldo, rows), make(out_ptr))
    r = _cached_map(("o", res_ptr, n_out, t_tok, ldo, rows), make(res_ptr)) if res_ptr else _NO_MAP
    return o, r


def partial_map(buf_ptr: int, n_out: int, t_tok: int, splits: int, bn: int) -> bytes | None:
    """TMA-store map of fp32 split-K slices [splits][t_tok][n_out]."""
    if (n_out * 4) % 16 or buf_ptr % 16:
        return None
    rows = min(bn, EPI_COLS)
    return _cached_map(("p", buf_ptr, n_out, t_tok, splits, rows),
                       lambda: core().make_tmap_3d(buf_ptr, _F32, n_out, t_tok, splits, n_out * 4,
                                                   t_tok * n_out * 4, BM, rows, 1, 0))


@dataclass
class Plan:
    bn: int
    splits: int
    grid: int
    swap: bool
    est_us: float = 0.0
    mt: int = 1  # 128-row A tiles per work unit (2 = two MMAs share each B tile)
    pf: int = 0  # k-blocks of L2 prefetch lead for streamed A tiles (0 = off)
    streamk: bool = False  # equal (tile, k-block) shares per CTA (fb_gemm_sk_*)
    pair: bool = False  # two-SM 256-row tiles (fb_gemm2_*); grid counts CTAs (two per pair)

    @property
    def kernel(self) -> str:
        if self.pair:
            return f"fb_gemm2_bf16_bn{self.bn}"
        return f"fb_gemm_sk_bn{self.bn}" if self.streamk else f"fb_gemm_bf16_bn{self.bn}_m{self.mt}"

    @property
    def smem(self) -> int:
        return smem_bytes_pair(self.bn) if self.pair else smem_bytes(self.bn, self.mt)

    @property
    def b_box(self) -> int:
        return self.bn // 2 if self.pair else self.bn


def plan(m_tok: int, n_out: int, k: int, sms: int | None = None, allow_split: bool = True,
         allow_streamk: bool = False, allow_pair: bool = True) -> Plan:
    """Chooses the tile width and split count with a small cost model:
    waves of CTAs x k-blocks per CTA x time per k-block, bounded below by the
    HBM time of the operands, plus the traffic of split slices."""
    sms = sms or _rt.sm_count()
    swap = m_tok <= 256
    mg, ng = (n_out, m_tok) if swap else (m_tok, n_out)
    kb = math.ceil(k / BK)
    tm = math.ceil(mg / BM)
    dram = (mg * k + ng * k) * 2 / _HBM_BPS
    best = None
    if swap:
        cands = [b for b in _BNS if b >= min(ng, 256) / 4 or b == 256]
    else:
        cands = [128, 256]
    # Measured: a CTA's TMA ring is latency bound - each stage takes about
    # (round-trip latency + MMA time) / ring depth - and two A tiles per unit
    # (mt=2) were never faster on decode shapes, so automatic plans use mt=1.
    for mt in (1,):
        tmm = math.ceil(mg / (BM * mt))
        for bn in cands:
            tn = math.ceil(ng / bn)
            stage = mt * BM * BK * 2 + bn * BK * 2
            stages = min(8, (192 * 1024) // stage)
            mma = mt * 2 * BM * bn * BK / _SM_MMA_FLOPS
            t_kb = max((_TMA_LATENCY + mma) / stages, stage / _CTA_FILL_BPS_MAX, mma)
            for s in range(1, (MAX_SPLITS if allow_split else 1) + 1):
                if s > 1 and kb // s < 4:
                    break
                units = tmm * tn * s
                waves = math.ceil(units / sms)
                kbp = math.ceil(kb / s)
                t = max(waves * (kbp * t_kb + 1.5e-6 * mt), dram)
                if s > 1:
                    t += 2 * s * mg * ng * 4 / _HBM_BPS
                if best is None or t < best.est_us * 1e-6 * 0.97:
                    best = Plan(bn=bn, splits=s, grid=min(units, sms), swap=swap, est_us=t * 1e6, mt=mt)
    # Streamed weight tiles (swap-AB decode GEMMs): an L2 prefetch 4 k-blocks
    # ahead of the shared-memory ring hides part of the DRAM latency
    # (measured 7-12% on Llama-3-8B decode shapes).
    if best.swap and kb >= 8:
        best.pf = 4
    # Stream-K: whole-tile plans whose tile count is not a multiple of the SM
    # count leave the last wave part empty; equal (tile, k-block) shares
    # remove that tail. Measured on B200 (Llama-3-8B gate_up, 224 tiles, both
    # with the TMA-store epilogue, CUDA-graph timed): 43.4 -> 35.0 us at 32
    # tokens (bn 32), 44.6 -> 38.3 us at 64 (bn 64), but 56.7 -> 68.0 us at
    # 256 (bn 256) and 77.0 us with bn 128, so only narrow tiles use it.
    if allow_pair and best.swap and mg >= 2 * BM and not (allow_streamk and best.bn <= 64):
        if _PAIR == "1" and best.bn >= 64:
            return pair_plan(mg, ng, k, best.bn, sms, allow_split, best.pf)
        if _PAIR == "auto" and ng >= 256:
            return pair_plan(mg, ng, k, 256, sms, allow_split, best.pf)
    if allow_streamk and best.swap and best.splits == 1 and best.mt == 1 and best.bn <= 64:
        tiles = math.ceil(mg / BM) * math.ceil(ng / best.bn)
        if tiles > sms and tiles % sms:
            best.streamk = True
            best.grid = sms
    return best


def pair_plan(mg: int, ng: int, k: int, bn: int, sms: int, allow_split: bool = True, pf: int = 4) -> Plan:
    """Two-SM plan for a swap-AB GEMM (mg weight rows, ng tokens): 256-row
    tiles, split K while more splits shorten the waves of CTA pairs."""
    pairs = sms // 2
    kb = math.ceil(k / BK)
    tiles = math.ceil(mg / (2 * BM)) * math.ceil(ng / bn)
    stage = BM * BK * 2 + (bn // 2) * BK * 2  # per SM
    stages = min(8, (192 * 1024) // stage)
    mma = 2 * BM * bn * BK / _SM_MMA_FLOPS
    t_kb = max((_TMA_LATENCY + mma) / stages, stage / _CTA_FILL_BPS_MAX, mma)
    dram = (mg * k + ng * k) * 2 / _HBM_BPS
    best_s, best_t = 1, None
    for s in range(1, (MAX_SPLITS if allow_split else 1) + 1):
        if s > 1 and kb // s < 4:
            break
        t = max(math.ceil(tiles * s / pairs) * math.ceil(kb / s) * t_kb, dram)
        if s > 1:
            t += 2 * s * mg * ng * 4 / _HBM_BPS
        if best_t is None or t < best_t * 0.97:
            best_s, best_t = s, t
    units = tiles * best_s
    return Plan(bn=bn, splits=best_s, grid=2 * min(units, pairs), swap=True, est_us=best_t * 1e6, pf=pf, pair=True)


# FOUNDRY_SWIGLU=0 turns the fused gate/up + SiLU*mul GEMM off (separate
# GEMM and silu_mul kernel, for comparison).
SWIGLU_ENABLED = os.environ.get("FOUNDRY_SWIGLU", "1") != "0"


def plan_swiglu(m_tok: int, inter: int, k: int, sms: int | None = None) -> Plan | None:
    """Plan of the fused gate/up GEMM + SiLU*mul (swap-AB, two 128-row A
    tiles per unit, no split-K since the epilogue is not linear in the sum);
    None when the shape does not allow it."""
    if not SWIGLU_ENABLED or m_tok > 256 or inter % BM:
        return None
    sms = sms or _rt.sm_count()
    kb = math.ceil(k / BK)
    tm = inter // BM
    dram = (2 * inter * k + m_tok * k) * 2 / _HBM_BPS
    best = None
    for bn in (32, 64, 128, 256):
        if bn < min(m_tok, 256) / 4 and bn != 256:
            continue
        units = tm * math.ceil(m_tok / bn)
        stage = 2 * BM * BK * 2 + bn * BK * 2
        stages = min(8, (192 * 1024) // stage)
        mma = 2 * 2 * BM * bn * BK / _SM_MMA_FLOPS
        t_kb = max((_TMA_LATENCY + mma) / stages, stage / _CTA_FILL_BPS_MAX, mma)
        t = max(math.ceil(units / sms) * (kb * t_kb + 3e-6), dram)
        if best is None or t < best.est_us * 1e-6 * 0.97:
            best = Plan(bn=bn, splits=1, grid=min(units, sms), swap=True, est_us=t * 1e6, mt=2,
                        pf=4 if kb >= 8 else 0)
    return best


# Stream-K form of the fused gate/up + SwiGLU GEMM (fb_gemm_swiglu_sk_bn256):
# for 129-256 tokens with fewer 128-feature units than SMs, every CTA takes
# an equal share of the (unit, k-block) iterations instead of one unit each.
# Off unless FOUNDRY_SWIGLU_SK=1. Measured on B200 at the Llama-3-8B decode
# shape (256 tokens, 14336 features = 112 units; CUDA graph of 20 launches,
# L2 flushed before each, programmatic dependent launch): 72.2 us against
# 62.1 us for the one-unit-per-CTA kernel on 112 SMs. A first version (fix-up
# reads straight from L2, accumulators held until the fp32 stores drained)
# took 78.3 us and the decode step 28.6k vs 30.1k tok/s; there every SM got
# the same MMA work (tensor pipe 50.5 % average, 51.1 % max) but CTAs that
# write one piece and read another ran up to 119.6k cycles against 75.8k:
# the fix-up costs more than the 36 idle SMs.
SWIGLU_SK_ENABLED = os.environ.get("FOUNDRY_SWIGLU_SK", "0") == "1"
SWIGLU_SK_BN = 256
SWIGLU_SK_MAXP = 3  # pieces of one unit (csrc/kernels/gemm_bf16.cu, SWIGLU_SK_MAXP)


@functools.lru_cache(maxsize=64)
def swiglu_sk_pieces(units: int, kb: int, grid: int) -> int:
    """Most CTAs that share one unit when ``grid`` CTAs split ``units * kb``
    iterations into ranges [T*b//grid, T*(b+1)//grid) (the kernel's split)."""
    total = units * kb
    start = [total * b // grid for b in range(grid + 1)]
    cta, worst = 0, 1
    for u in range(units):
        lo, hi = u * kb, u * kb + kb - 1
        while start[cta + 1] <= lo:
            cta += 1
        last = cta
        while start[last + 1] <= hi:
            last += 1
        worst = max(worst, last - cta + 1)
    return worst


def swiglu_sk_sizes(inter: int) -> tuple[int, int]:
    """(fp32 workspace elements, int32 flag words) of the stream-K SwiGLU
    GEMM for ``inter`` features per rank."""
    units = inter // BM
    return units * SWIGLU_SK_MAXP * 2 * BM * SWIGLU_SK_BN, units * (1 + SWIGLU_SK_MAXP)


def plan_swiglu_sk(m_tok: int, inter: int, k: int, sms: int | None = None, force: bool = False) -> Plan | None:
    """Stream-K plan of the fused gate/up GEMM, or None where it does not
    apply: switched off (``force`` ignores FOUNDRY_SWIGLU_SK), tokens outside
    129..256, as many units as SMs or more (the one-unit-per-CTA kernel then
    fills the GPU), or a split that would cut a unit into more than
    SWIGLU_SK_MAXP pieces."""
    if not (force or (SWIGLU_ENABLED and SWIGLU_SK_ENABLED)) or not 128 < m_tok <= SWIGLU_SK_BN or inter % BM:
        return None
    sms = sms or _rt.sm_count()
    units, kb = inter // BM, math.ceil(k / BK)
    if units >= sms or units * kb < sms or swiglu_sk_pieces(units, kb, sms) > SWIGLU_SK_MAXP:
        return None
    return Plan(bn=SWIGLU_SK_BN, splits=1, grid=sms, swap=True, mt=2, pf=4 if kb >= 8 else 0, streamk=True)


def linear_swiglu(x: torch.Tensor, w_gu: torch.Tensor, out: torch.Tensor,
                  plan_override: Plan | None = None, sk: StreamKBuffer | None = None) -> torch.Tensor | None:
    """out = silu(x @ gate.T) * (x @ up.T) in one GEMM, where w_gu is [gate;
    up] ([2 * I, K], gate rows first) and out is [T, I] bf16. Returns None
    (nothing launched) when the shape has no fused plan: more than 256 tokens,
    I not a multiple of 128, or rows the TMA stores cannot address. With a
    workspace ``sk`` (``swiglu_sk_sizes``; flags zero before the first launch,
    left zero by every launch) and FOUNDRY_SWIGLU_SK=1, shapes with fewer
    units than SMs run the stream-K kernel (or pass its plan as
    ``plan_override``)."""
    t_tok, k = x.shape
    two_i, k2 = w_gu.shape
    inter = two_i // 2
    assert k == k2 and out.shape == (t_tok, inter) and out.stride(1) == 1
    p = plan_override
    if p is None and sk is not None:
        p = plan_swiglu_sk(t_tok, inter, k)
        ws_n, fl_n = swiglu_sk_sizes(inter)
        if p is not None and (sk.ws.numel() < ws_n or sk.flags.numel() < fl_n):
            p = None
    if p is None:
        p = plan_swiglu(t_tok, inter, k)
    if p is None:
        return None
    om = out_maps(out.data_ptr(), 0, inter, t_tok, out.stride(0), p.bn)
    if om is None:
        return None
    mode = EPI_TRANSPOSE | EPI_TMA_OUT | EPI_SWIGLU | ((min(p.pf, 255) & 0xFF) << 8)
    if math.ceil(t_tok / p.bn) == 1:
        mode |= EPI_A_STREAM
    if _rt.pdl_active():
        mode |= EPI_A_CONST
    if p.streamk:
        assert sk is not None and p.bn == SWIGLU_SK_BN and t_tok <= p.bn
        args = [tmap(w_gu, BM), tmap(x, p.bn), om[0], two_i, t_tok, k, mode, sk.ws.data_ptr(), sk.flags.data_ptr()]
        _rt.launch("gemm_bf16", f"fb_gemm_swiglu_sk_bn{p.bn}", (p.grid,), (192,), args, smem=smem_bytes(p.bn, 2))
        return out
    args = [tmap(w_gu, BM), tmap(x, p.bn), om[0], _NO_MAP, out.data_ptr(), 0, two_i, t_tok, k, out.stride(0), mode,
            1, 0, 0]
    _rt.launch("gemm_bf16", p.kernel, (p.grid,), (192,), args, smem=p.smem)
    return out


def linear_multicast(x: torch.Tensor, w: torch.Tensor, target: int, plan_override: Plan | None = None) -> None:
    """x @ w.T written by the GEMM epilogue straight to ``target``, an NVLS
    multicast address: every tile lands in the same slot of every rank's
    buffer as soon as it is computed (the GEMM half of a fused all-reduce)."""
    t_tok, k = x.shape
    n_out = w.shape[0]
    p = plan_override or plan(t_tok, n_out, k, allow_split=False, allow_pair=False)
    assert p.splits == 1 and not p.pair
    if p.swap:
        a, b, mg, ng, mode = w, x, n_out, t_tok, EPI_TRANSPOSE | EPI_MCAST
    else:
        a, b, mg, ng, mode = x, w, t_tok, n_out, EPI_MCAST
    args = [tmap(a, BM), tmap(b, p.bn), _NO_MAP, _NO_MAP, target, 0, mg, ng, k, n_out, mode, 1, 0, 0]
    _rt.launch("gemm_bf16", p.kernel, (p.grid,), (192,), args, smem=smem_bytes(p.bn, p.mt))


def linear(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None,
           residual: torch.Tensor | None = None, partials: PartialBuffer | None = None,
           plan_override: Plan | None = None, streamk: StreamKBuffer | None = None):
    """out = x @ w.T (+ residual). x: [T, K] bf16, w: [N, K] bf16, out: [T, N] bf16.

    Returns ``out`` - or, when ``partials`` is given and the plan splits K, a
    ``Partial`` whose slices the caller's next op must consume (``residual``
    is then NOT applied; the consumer adds it). ``residual`` may alias ``out``.
    """
    assert x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16
    t_tok, k = x.shape
    n_out, k2 = w.shape
    assert k == k2, f"K mismatch {k} vs {k2}"
    p = plan_override or plan(t_tok, n_out, k, allow_split=partials is not None, allow_streamk=streamk is not None)
    sk_maps = None
    if p.streamk and streamk is not None and streamk.fits(p.grid, p.bn) and out is not None:
        sk_maps = out_maps(out.data_ptr(), residual.data_ptr() if residual is not None else 0, n_out, t_tok,
                           out.stride(0), p.bn)
    if p.streamk and sk_maps is None:  # no workspace, or rows the TMA stores cannot address
        p = plan(t_tok, n_out, k, allow_split=partials is not None)
    mode = 0
    if p.swap:
        a, b, mg, ng = w, x, n_out, t_tok
        mode |= EPI_TRANSPOSE
        if math.ceil(ng / p.bn) == 1:
            mode |= EPI_A_STREAM  # each weight byte is read once: evict-first
        if _rt.pdl_active():
            mode |= EPI_A_CONST  # inside the decode step no kernel writes the weights
    else:
        a, b, mg, ng = x, w, t_tok, n_out
    mode |= (min(p.pf, 255) & 0xFF) << 8
    if p.splits > 1:
        assert partials is not None
        need = p.splits * t_tok * n_out
        if need > partials.numel:
            raise RuntimeError(f"split-K slice buffer too small: need {need} floats, have {partials.numel}")
        pm = partial_map(partials.buf.data_ptr(), n_out, t_tok, p.splits, p.bn) if p.swap else None
        if pm is not None:
            mode |= EPI_TMA_OUT
        maps = [pm or _NO_MAP, _NO_MAP]
        args = [tmap(a, BM), tmap(b, p.b_box), *maps, 0, 0, mg, ng, k, n_out, mode, p.splits,
                partials.buf.data_ptr(), t_tok * n_out]
        _rt.launch("gemm_bf16", p.kernel, (p.grid,), (192,), args, smem=p.smem)
        return Partial(partials.buf, p.splits, t_tok, n_out)
    if out is None:
        out = torch.empty(t_tok, n_out, dtype=torch.bfloat16, device=x.device)
    assert out.stride(1) == 1 and out.shape == (t_tok, n_out)
    if residual is not None:
        assert residual.shape == out.shape and residual.stride() == out.stride()
        mode |= EPI_RESIDUAL
    if p.streamk:
        # A tile may be split between two neighbouring CTAs only: stream-K
        # needs at least one whole tile per CTA.
        if math.ceil(mg / BM) * math.ceil(ng / p.bn) < p.grid:
            raise ValueError(f"stream-K plan has fewer tiles than its {p.grid} CTAs")
        args = [tmap(a, BM), tmap(b, p.bn), *sk_maps, mg, ng, k, mode | EPI_TMA_OUT, streamk.ws.data_ptr(),
                streamk.flags.data_ptr()]
        _rt.launch("gemm_bf16", p.kernel, (p.grid,), (192,), args, smem=smem_bytes(p.bn, 1))
        return out
    om = None
    if p.swap:
        om = out_maps(out.data_ptr(), residual.data_ptr() if residual is not None else 0, n_out, t_tok,
                      out.stride(0), p.bn)
    if om is not None:
        mode |= EPI_TMA_OUT
    maps = list(om) if om is not None else [_NO_MAP, _NO_MAP]
    args = [tmap(a, BM), tmap(b, p.b_box), *maps, out.data_ptr(), residual.data_ptr() if residual is not None else 0,
            mg, ng, k, out.stride(0), mode, 1, 0, 0]
    _rt.launch("gemm_bf16", p.kernel, (p.grid,), (192,), args, smem=p.smem)
    return out
