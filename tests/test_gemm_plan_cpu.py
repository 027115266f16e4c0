"""The bf16 GEMM planner (foundry_b200/ops/gemm.py) on CPU: every plan names
a kernel the image exports, fits the launch limits, and keeps the invariants
the kernels rely on (split-K only with enough k-blocks per split, even grids
of CTA pairs for the two-SM tiles, swap-AB only for decode-sized batches)."""

import os
import re

import pytest

from foundry_b200.ops import gemm as G

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SHAPES = [(t, n, k) for t in (1, 7, 16, 64, 128, 200, 256, 300, 1024, 2048)
          for (n, k) in ((6144, 4096), (4096, 4096), (28672, 4096), (4096, 14336), (128256, 4096),
                         (5120, 2048), (2048, 4096), (640, 512), (384, 1024))]


def _exported_kernels():
    src = open(os.path.join(ROOT, "csrc", "kernels", "gemm_bf16.cu")).read()
    names = set()
    for bn, mt in re.findall(r"^FB_GEMM_INSTANCE\((\d+), (\d+)\)", src, re.M):
        names.add(f"fb_gemm_bf16_bn{bn}_m{mt}")
    for bn in re.findall(r"^FB_GEMM_SK_INSTANCE\((\d+)\)", src, re.M):
        names.add(f"fb_gemm_sk_bn{bn}")
    for bn in re.findall(r"^FB_GEMM_PAIR_INSTANCE\((\d+)\)", src, re.M):
        names.add(f"fb_gemm2_bf16_bn{bn}")
    return names


KERNELS = _exported_kernels()


@pytest.mark.parametrize("t,n,k", SHAPES)
def test_plans_are_launchable(t, n, k):
    for allow_split in (False, True):
        for allow_streamk in (False, True):
            p = G.plan(t, n, k, sms=148, allow_split=allow_split, allow_streamk=allow_streamk)
            assert p.kernel in KERNELS, p
            assert p.swap == (t <= 256)
            assert 1 <= p.splits <= (G.MAX_SPLITS if allow_split else 1)
            kb = -(-k // G.BK)
            assert p.splits == 1 or kb // p.splits >= 4
            assert 1 <= p.grid <= 148
            assert p.smem <= 227 * 1024
            if p.streamk:
                assert allow_streamk and p.bn <= 64 and p.splits == 1


@pytest.mark.parametrize("t,n,k", [s for s in SHAPES if s[0] <= 256 and s[1] >= 256])
def test_pair_plans_are_launchable(t, n, k):
    one = G.plan(t, n, k, sms=148)
    p = G.pair_plan(n, t, k, max(64, one.bn), 148)
    assert p.pair and p.kernel in KERNELS, p
    assert p.grid % 2 == 0 and 2 <= p.grid <= 148
    tiles = -(-n // 256) * -(-t // p.bn)
    assert p.grid == 2 * min(tiles * p.splits, 74)
    assert p.b_box == p.bn // 2 and p.smem <= 227 * 1024
    kb = -(-k // G.BK)
    assert p.splits == 1 or kb // p.splits >= 4


def test_pair_tile_policy():
    """Default ("auto"): two-SM tiles, 256 tokens wide, exactly for swap-AB
    plans of 256-token batches with at least 256 weight rows; never when the
    caller cannot take them (multicast / all-reduce epilogues)."""
    assert G._PAIR == os.environ.get("FOUNDRY_GEMM_PAIR", "auto")
    for (t, n, k) in SHAPES:
        assert not G.plan(t, n, k, sms=148, allow_pair=False).pair
        if G._PAIR == "auto":
            p = G.plan(t, n, k, sms=148)
            assert p.pair == (t == 256 and n >= 256), (t, n, k, p)
            if p.pair:
                assert p.bn == 256 and p.kernel in KERNELS
        elif G._PAIR == "0":
            assert not any(G.plan(t, n, k, sms=148).pair for (t, n, k) in SHAPES)


def _pieces_brute(units, kb, grid):
    """Pieces per unit by walking every iteration (the kernel's ranges)."""
    total = units * kb
    owner = [max(b for b in range(grid) if total * b // grid <= i) for i in range(total)]
    return max(len(set(owner[u * kb:(u + 1) * kb])) for u in range(units))


@pytest.mark.parametrize("units,kb,grid", [(112, 64, 148), (96, 16, 148), (76, 32, 148), (140, 64, 148), (28, 128, 148),
                                           (112, 64, 147), (10, 8, 37)])
def test_swiglu_streamk_pieces(units, kb, grid):
    """The host's count of CTAs sharing one unit matches a walk over the
    kernel's iteration ranges; the plan exists only when it stays within the
    kernel's slot count, and names an exported kernel."""
    assert G.swiglu_sk_pieces(units, kb, grid) == _pieces_brute(units, kb, grid)
    src = open(os.path.join(ROOT, "csrc", "kernels", "gemm_bf16.cu")).read()
    assert f"constexpr int SWIGLU_SK_MAXP = {G.SWIGLU_SK_MAXP};" in src
    assert re.search(rf"^FB_GEMM_SWIGLU_SK_INSTANCE\({G.SWIGLU_SK_BN}\)", src, re.M)
    p = G.plan_swiglu_sk(256, units * G.BM, kb * G.BK, sms=grid, force=True)
    ok = units < grid and units * kb >= grid and G.swiglu_sk_pieces(units, kb, grid) <= G.SWIGLU_SK_MAXP
    assert (p is not None) == ok
    if p is not None:
        assert p.streamk and p.mt == 2 and p.grid == grid and p.bn == G.SWIGLU_SK_BN
    # off unless asked for: the default plan never picks it
    if not G.SWIGLU_SK_ENABLED:
        assert G.plan_swiglu_sk(256, units * G.BM, kb * G.BK, sms=grid) is None
    ws_n, fl_n = G.swiglu_sk_sizes(units * G.BM)
    assert ws_n == units * G.SWIGLU_SK_MAXP * 2 * G.BM * G.SWIGLU_SK_BN and fl_n == units * (1 + G.SWIGLU_SK_MAXP)
