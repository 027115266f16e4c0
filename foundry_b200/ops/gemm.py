"""bf16 linear layers on the tcgen05 GEMM (csrc/kernels/gemm_bf16.cu).

``linear(x, w)`` computes ``x @ w.T`` (nn.Linear layout: ``w`` is
[out_features, in_features]). Small token counts (decode) run "swap-AB": the
weight rows fill the 128-row MMA M dimension and the tokens become the MMA N
dimension (16..256), the output is written transposed back to [tokens, out].
Narrow problems are split along K so every SM streams weights; split partials
are reduced deterministically inside the kernel.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from .._native import core
from . import _rt

BM, BK = 128, 64
EPI_TRANSPOSE, EPI_RESIDUAL, EPI_A_STREAM, EPI_B_STREAM = 1, 2, 4, 8
_BF16 = 9  # CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
_SWIZZLE_128B = 3
_BNS = (16, 32, 64, 128, 256)


def smem_bytes(bn: int) -> int:
    stage = BM * BK * 2 + bn * BK * 2
    stages = min(8, (200 * 1024) // stage)
    return stages * stage + 1024 + 256


class GemmWorkspace:
    """Split-K partial tiles (fp32) and per-tile arrival counters.

    Counters must start at zero; the kernel re-arms them, so a workspace can be
    reused by any number of launches and graph replays, but not by two GEMMs
    running concurrently.
    """

    def __init__(self, nbytes: int = 64 << 20, n_counters: int = 1 << 16, device=None,
                 ws: torch.Tensor | None = None, counters: torch.Tensor | None = None):
        device = device or torch.device("cuda", torch.cuda.current_device())
        self.ws = ws if ws is not None else torch.empty(nbytes // 4, dtype=torch.float32, device=device)
        self.counters = counters if counters is not None else torch.zeros(n_counters, dtype=torch.int32, device=device)

    @property
    def nbytes(self) -> int:
        return self.ws.numel() * 4


_default_ws: dict[int, GemmWorkspace] = {}


def default_workspace() -> GemmWorkspace:
    dev = torch.cuda.current_device()
    ws = _default_ws.get(dev)
    if ws is None:
        ws = _default_ws[dev] = GemmWorkspace()
    return ws


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
        if len(_tmaps) > 4096:
            _tmaps.clear()
        _tmaps[key] = m
    return m


@dataclass
class Plan:
    bn: int
    splits: int
    grid: int
    swap: bool


def plan(m_tok: int, n_out: int, k: int, sms: int | None = None) -> Plan:
    sms = sms or _rt.sm_count()
    swap = m_tok <= 256
    if swap:
        mg, ng = n_out, m_tok
        bn = next(b for b in _BNS if b >= ng)
    else:
        mg, ng = m_tok, n_out
        bn = 256 if ng >= 256 else next(b for b in _BNS if b >= ng)
    tiles = math.ceil(mg / BM) * math.ceil(ng / bn)
    kb = math.ceil(k / BK)
    splits = 1
    if tiles < sms:
        splits = max(1, min(math.ceil(sms / tiles), kb // 4, 16))
    grid = min(tiles * splits, sms)
    return Plan(bn=bn, splits=splits, grid=grid, swap=swap)


def linear(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None,
           residual: torch.Tensor | None = None, ws: GemmWorkspace | None = None,
           plan_override: Plan | None = None) -> torch.Tensor:
    """out = x @ w.T (+ residual). x: [T, K] bf16, w: [N, K] bf16, out: [T, N] bf16.

    ``residual`` may alias ``out`` (in-place residual add).
    """
    assert x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16
    t_tok, k = x.shape
    n_out, k2 = w.shape
    assert k == k2, f"K mismatch {k} vs {k2}"
    if out is None:
        out = torch.empty(t_tok, n_out, dtype=torch.bfloat16, device=x.device)
    assert out.stride(1) == 1 and out.shape == (t_tok, n_out)
    p = plan_override or plan(t_tok, n_out, k)
    ws = ws or default_workspace()
    mode = 0
    if p.swap:
        a, b, mg, ng = w, x, n_out, t_tok
        mode |= EPI_TRANSPOSE | EPI_A_STREAM
    else:
        a, b, mg, ng = x, w, t_tok, n_out
    if residual is not None:
        assert residual.shape == out.shape and residual.stride() == out.stride()
        mode |= EPI_RESIDUAL
    if p.splits > 1:
        need = math.ceil(mg / BM) * math.ceil(ng / p.bn) * p.splits * BM * p.bn * 4
        if need > ws.nbytes:
            raise RuntimeError(f"GEMM workspace too small: need {need} bytes, have {ws.nbytes}")
        if math.ceil(mg / BM) * math.ceil(ng / p.bn) > ws.counters.numel():
            raise RuntimeError("GEMM workspace has too few tile counters")
    args = [
        tmap(a, BM), tmap(b, p.bn), out.data_ptr(),
        residual.data_ptr() if residual is not None else 0,
        mg, ng, k, out.stride(0), mode, p.splits, ws.ws.data_ptr(), ws.counters.data_ptr(),
    ]
    _rt.launch("gemm_bf16", f"fb_gemm_bf16_bn{p.bn}", (p.grid,), (192,), args, smem=smem_bytes(p.bn))
    return out
