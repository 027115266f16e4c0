"""Numerics of the sm_100a kernels against plain PyTorch fp32 references."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _bf(*shape, scale=1.0, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(*shape, generator=g, device="cuda") * scale).to(torch.bfloat16)


@pytest.fixture(autouse=True)
def _status_clean():
    from foundry_b200 import ops

    yield
    for img in ("gemm_bf16", "elementwise", "attention"):
        if img in ops._rt.loaded_images():
            assert ops.status(img) == 0, f"{img} reported a device-side error"


@pytest.mark.parametrize("t,n,k", [
    (1, 512, 256), (7, 384, 512), (16, 6144, 4096), (100, 1024, 1024), (256, 4096, 4096),
    (300, 1024, 512), (512, 2048, 1024), (1000, 768, 2048),
])
def test_linear(t, n, k):
    from foundry_b200 import ops

    x = _bf(t, k, seed=1)
    w = _bf(n, k, scale=0.05, seed=2)
    out = ops.linear(x, w)
    ref = x.float() @ w.float().T
    torch.testing.assert_close(out.float(), ref, atol=2e-2 * math.sqrt(k / 256), rtol=2e-2)


@pytest.mark.parametrize("bn,mt,splits", [(16, 1, 1), (64, 2, 1), (128, 2, 3), (256, 2, 1), (256, 1, 2), (32, 2, 4)])
@pytest.mark.parametrize("t,n,k,swap", [(24, 1152, 1024, True), (300, 640, 512, False)])
def test_linear_all_tile_configs(bn, mt, splits, t, n, k, swap):
    """Every kernel variant (tile width x A tiles per unit x split) against fp32."""
    from foundry_b200 import ops
    from foundry_b200.ops.gemm import Plan

    if not swap and bn < 128:
        pytest.skip("prefill path uses 128/256-wide tiles")
    x = _bf(t, k, seed=21)
    w = _bf(n, k, scale=0.05, seed=22)
    p = Plan(bn=bn, splits=splits, grid=min(148, 64), swap=swap, mt=mt)
    ref = x.float() @ w.float().T
    if splits == 1:
        out = ops.linear(x, w, plan_override=p)
        torch.testing.assert_close(out.float(), ref, atol=4e-2, rtol=2e-2)
    else:
        pb = ops.PartialBuffer(splits * t * n)
        r = ops.linear(x, w, partials=pb, plan_override=p)
        total = r.buf[: splits * t * n].view(splits, t, n).sum(0)
        torch.testing.assert_close(total, ref, atol=4e-2, rtol=2e-2)


@pytest.mark.parametrize("bn,splits,t,n,k,residual", [
    (64, 1, 64, 512, 256, False), (128, 2, 200, 4224, 4160, True), (256, 1, 256, 2304, 1024, True),
    (256, 3, 256, 1536, 4096, False),
])
def test_linear_pair_tiles(bn, splits, t, n, k, residual):
    """Two-SM (cta_group::2) 256-row tiles against fp32: M, N and K tails,
    residual epilogue and split-K slices."""
    from foundry_b200 import ops
    from foundry_b200.ops import gemm as G

    x = _bf(t, k, seed=31)
    w = _bf(n, k, scale=0.05, seed=32)
    p = G.pair_plan(n, t, k, bn, G._rt.sm_count(), allow_split=splits > 1)
    p.splits = splits
    p.grid = 2 * min(math.ceil(n / 256) * math.ceil(t / bn) * splits, G._rt.sm_count() // 2)
    assert p.pair and p.kernel == f"fb_gemm2_bf16_bn{bn}"
    ref = x.float() @ w.float().T
    if splits > 1:
        pb = ops.PartialBuffer(splits * t * n)
        r = ops.linear(x, w, partials=pb, plan_override=p)
        total = r.buf[: splits * t * n].view(splits, t, n).sum(0)
        torch.testing.assert_close(total, ref, atol=4e-2, rtol=2e-2)
        return
    res = _bf(t, n, seed=33) if residual else None
    out = res.clone() if residual else torch.empty(t, n, dtype=torch.bfloat16, device="cuda")
    ops.linear(x, w, out=out, residual=out if residual else None, plan_override=p)
    want = ref + (res.float() if residual else 0)
    torch.testing.assert_close(out.float(), want, atol=4e-2, rtol=2e-2)


@pytest.mark.parametrize("t,n,k", [(8, 4096, 4096), (64, 1024, 14336), (600, 512, 1024)])
def test_linear_residual(t, n, k):
    from foundry_b200 import ops

    x = _bf(t, k, seed=3)
    w = _bf(n, k, scale=0.02, seed=4)
    h = _bf(t, n, seed=5)
    ref = h.float() + x.float() @ w.float().T
    out = ops.linear(x, w, out=h, residual=h)
    assert out.data_ptr() == h.data_ptr()
    torch.testing.assert_close(out.float(), ref, atol=5e-2, rtol=2e-2)


@pytest.mark.parametrize("t,n,k", [(32, 1024, 4096), (256, 4096, 4096), (256, 4096, 14336), (7, 6144, 4096)])
def test_linear_split_partials(t, n, k):
    """Split-K GEMMs return fp32 slices; consumers sum them (deterministically)."""
    from foundry_b200 import ops

    x = _bf(t, k, seed=6)
    w = _bf(n, k, scale=0.02, seed=7)
    pb = ops.PartialBuffer(8 * t * n)
    p = ops.plan(t, n, k, allow_split=True)
    assert p.splits > 1, p
    r = ops.linear(x, w, partials=pb)
    assert isinstance(r, ops.Partial) and r.splits == p.splits
    total = r.buf[: r.splits * r.stride].view(r.splits, t, n).sum(0)
    torch.testing.assert_close(total, x.float() @ w.float().T, atol=2e-2 * math.sqrt(k / 256), rtol=2e-2)
    # consumer: fused residual add + RMSNorm
    h = _bf(t, n, seed=8)
    h0 = h.clone()
    wn = _bf(n, seed=9)
    xo = torch.empty_like(h)
    ops.add_rmsnorm_partials(r, h, wn, xo, 1e-5)
    href = (total + h0.float()).to(torch.bfloat16)
    # fp32 summation order differs from torch's reduction: allow one bf16 ulp
    torch.testing.assert_close(h.float(), href.float(), atol=1e-2, rtol=8e-3)
    hf = href.float()
    ref = hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-5) * wn.float()
    torch.testing.assert_close(xo.float(), ref, atol=2e-2, rtol=1e-2)
    # determinism: the same launch twice gives identical slices
    s1 = r.buf[: r.splits * r.stride].clone()
    ops.linear(x, w, partials=pb)
    assert torch.equal(s1, pb.buf[: r.splits * r.stride])


def test_rmsnorm_silu_embedding_argmax():
    from foundry_b200 import ops

    x = _bf(33, 4096, seed=8)
    w = _bf(4096, seed=9)
    out = torch.empty_like(x)
    ops.rmsnorm(x, w, out, 1e-5)
    xf = x.float()
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5) * w.float()
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=1e-2)

    gu = _bf(17, 2 * 1024, seed=10)
    act = torch.empty(17, 1024, dtype=torch.bfloat16, device="cuda")
    ops.silu_mul(gu, act)
    g, u = gu.float()[:, :1024], gu.float()[:, 1024:]
    torch.testing.assert_close(act.float(), torch.nn.functional.silu(g) * u, atol=2e-2, rtol=1e-2)

    table = _bf(1000, 256, seed=11)
    ids = torch.randint(0, 1000, (9,), device="cuda", dtype=torch.int32)
    emb = torch.empty(9, 256, dtype=torch.bfloat16, device="cuda")
    ops.embedding(ids, table, emb)
    assert torch.equal(emb, table[ids.long()])

    logits = _bf(5, 128256, seed=12)
    am = torch.empty(5, dtype=torch.int32, device="cuda")
    ops.argmax(logits, am)
    assert torch.equal(am.long(), logits.float().argmax(-1))


def test_init_normal_deterministic():
    from foundry_b200 import ops

    a = torch.empty(1 << 20, dtype=torch.bfloat16, device="cuda")
    b = torch.empty_like(a)
    ops.init_normal_(a, seed=123, std=0.02)
    ops.init_normal_(b, seed=123, std=0.02)
    assert torch.equal(a, b)
    assert abs(a.float().std().item() - 0.02) < 1e-3
    assert abs(a.float().mean().item()) < 1e-3


@pytest.mark.parametrize("qk_norm", [False, True])
def test_rope_kv_write(qk_norm):
    from foundry_b200 import ops

    t, nq, nkv, d, page = 10, 8, 2, 128, 64
    qkv = _bf(t, (nq + 2 * nkv) * d, seed=13)
    pos = torch.tensor([0, 1, 2, 63, 64, 65, 100, 5, 7, 200], dtype=torch.int32, device="cuda")
    cs = ops.rope_cos_sin(256, 500000.0, device="cuda")
    q_out = torch.empty(t, nq, d, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(8, nkv, page, d, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    slots = torch.arange(t, dtype=torch.int32, device="cuda") * 37 % (8 * page)
    qn = _bf(d, seed=14) if qk_norm else None
    kn = _bf(d, seed=15) if qk_norm else None
    k_out = torch.empty(t, nkv, d, dtype=torch.bfloat16, device="cuda")
    ops.rope_kv_write(qkv, pos, cs, q_out, kc, vc, slots, nq, nkv, qn, kn, 1e-6, k_out=k_out)

    f = qkv.float()
    q = f[:, : nq * d].view(t, nq, d)
    k = f[:, nq * d:(nq + nkv) * d].view(t, nkv, d)
    v = f[:, (nq + nkv) * d:].view(t, nkv, d)
    if qk_norm:
        q = q * torch.rsqrt(q.pow(2).mean(-1, keepdim=True) + 1e-6) * qn.float()
        k = k * torch.rsqrt(k.pow(2).mean(-1, keepdim=True) + 1e-6) * kn.float()
    c = cs[pos.long(), :, 0][:, None, :]
    s = cs[pos.long(), :, 1][:, None, :]

    def rot(x):
        return torch.cat([x[..., :64] * c - x[..., 64:] * s, x[..., 64:] * c + x[..., :64] * s], -1)

    torch.testing.assert_close(q_out.float(), rot(q), atol=3e-2, rtol=2e-2)
    torch.testing.assert_close(k_out.float(), rot(k), atol=3e-2, rtol=2e-2)
    for i in range(t):
        sl = int(slots[i])
        torch.testing.assert_close(kc[sl // page, :, sl % page].float(), rot(k)[i], atol=3e-2, rtol=2e-2)
        assert torch.equal(vc[sl // page, :, sl % page], qkv[i, (nq + nkv) * d:].view(nkv, d))


def _ref_decode(q, kc, vc, tables, lens, page=64):
    b, nq, d = q.shape
    nkv = kc.shape[1]
    g = nq // nkv
    out = torch.empty(b, nq, d, device=q.device)
    for i in range(b):
        n = int(lens[i])
        pages = tables[i, : math.ceil(n / page)].long()
        k = kc[pages].permute(0, 2, 1, 3).reshape(-1, nkv, d)[:n].float()
        v = vc[pages].permute(0, 2, 1, 3).reshape(-1, nkv, d)[:n].float()
        k = k.repeat_interleave(g, 1)
        v = v.repeat_interleave(g, 1)
        att = torch.einsum("hd,shd->hs", q[i].float(), k) / math.sqrt(d)
        out[i] = torch.einsum("hs,shd->hd", att.softmax(-1), v)
    return out


@pytest.mark.parametrize("impl", ["tc1", "tc3", "simt"])
@pytest.mark.parametrize("b,nq,nkv,lens", [
    (3, 32, 8, [1, 64, 130]), (5, 64, 8, [640, 17, 333, 64, 65]), (2, 32, 4, [700, 2]),
    (64, 32, 8, None), (300, 32, 8, None),
])
def test_decode_attention(b, nq, nkv, lens, impl):
    from foundry_b200 import ops

    page, d = 64, 128
    max_pages = 12
    nb = b * max_pages
    kc = _bf(nb, nkv, page, d, seed=16)
    vc = _bf(nb, nkv, page, d, seed=17)
    q = _bf(b, nq, d, seed=18)
    if lens is None:
        lens = [1 + (37 * i) % (max_pages * page) for i in range(b)]
    lens_t = torch.tensor(lens, dtype=torch.int32, device="cuda")
    perm = torch.randperm(nb, generator=torch.Generator().manual_seed(0)).to(torch.int32).cuda()
    tables = perm.view(b, max_pages).contiguous()
    ws = ops.DecodeWorkspace(b, nq, 16)
    out = torch.empty(b, nq, d, dtype=torch.bfloat16, device="cuda")
    ref = _ref_decode(q, kc, vc, tables, lens_t)
    for splits in (None, (1, max_pages), (3, 4) if impl.startswith("tc") else (4, 3)):
        out.zero_()
        ops.decode_attention(q, kc, vc, tables, lens_t, out, max_pages, ws, splits=splits, impl=impl)
        torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("impl", ["tc1", "tc3", "simt"])
def test_decode_attention_ignores_nan_past_end(impl):
    """Cache slots past a sequence's length may hold anything (here NaN)."""
    from foundry_b200 import ops

    b, nq, nkv, page, d, max_pages = 4, 32, 8, 64, 128, 6
    nb = b * max_pages
    kc = _bf(nb, nkv, page, d, seed=30)
    vc = _bf(nb, nkv, page, d, seed=31)
    lens = [1, 70, 129, 300]
    tables = torch.arange(nb, dtype=torch.int32, device="cuda").view(b, max_pages)
    for i, n in enumerate(lens):
        for p in range(max_pages):
            lo = max(0, n - p * page)
            if lo < page:
                kc[tables[i, p], :, lo:] = float("nan")
                vc[tables[i, p], :, lo:] = float("nan")
    q = _bf(b, nq, d, seed=32)
    lens_t = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = torch.empty(b, nq, d, dtype=torch.bfloat16, device="cuda")
    ops.decode_attention(q, kc, vc, tables, lens_t, out, max_pages, ops.DecodeWorkspace(b, nq, 8), impl=impl)
    assert torch.isfinite(out.float()).all()
    ref = _ref_decode(q, kc, vc, tables, lens_t)
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("impl,nq,nkv,seqlens", [
    ("simt", 8, 2, [1, 70, 129, 64]), ("tc", 8, 2, [1, 70, 129, 64]), ("tc", 16, 2, [300, 5, 256, 128, 513]),
    ("tc", 32, 8, [1000])])
def test_prefill_attention(impl, nq, nkv, seqlens):
    from foundry_b200 import ops
    from foundry_b200.ops.attention import PREFILL_TILE

    d = 128
    t = sum(seqlens)
    q = _bf(t, nq * d, seed=19)
    k = _bf(t, nkv * d, seed=20)
    v = _bf(t, nkv * d, seed=21)
    cu = torch.tensor([0] + list(torch.tensor(seqlens).cumsum(0)), dtype=torch.int32, device="cuda")
    ts, tst = ops.prefill_tiles(seqlens, PREFILL_TILE[impl])
    out = torch.full((t, nq * d), float("nan"), dtype=torch.bfloat16, device="cuda")
    ops.prefill_attention(q, k, v, out, cu, torch.tensor(ts, dtype=torch.int32, device="cuda"),
                          torch.tensor(tst, dtype=torch.int32, device="cuda"), nq, nkv, impl=impl)
    assert ops.status("prefill_tc" if impl == "tc" else "attention") == 0
    g = nq // nkv
    off = 0
    for n in seqlens:
        qq = q[off:off + n].float().view(n, nq, d)
        kk = k[off:off + n].float().view(n, nkv, d).repeat_interleave(g, 1)
        vv = v[off:off + n].float().view(n, nkv, d).repeat_interleave(g, 1)
        att = torch.einsum("thd,shd->hts", qq, kk) / math.sqrt(d)
        mask = torch.triu(torch.ones(n, n, dtype=torch.bool, device="cuda"), 1)
        ref = torch.einsum("hts,shd->thd", att.masked_fill(mask, float("-inf")).softmax(-1), vv)
        torch.testing.assert_close(out[off:off + n].float().view(n, nq, d), ref, atol=2e-2, rtol=2e-2)
        off += n


@pytest.mark.parametrize("t,n,k", [(64, 28672, 4096), (16, 28672, 4096), (40, 19000, 1024), (64, 40000, 512)])
def test_linear_streamk(t, n, k):
    """Stream-K decode GEMM (tiles split between neighbouring CTAs, fp32
    partials met through a workspace): matches fp32, with and without the
    residual epilogue, on repeated launches (the tickets reset themselves)
    and bit-identically across launches."""
    from foundry_b200 import ops
    from foundry_b200.ops.gemm import plan

    p = plan(t, n, k, allow_streamk=True)
    assert p.streamk, p
    x = _bf(t, k, seed=31)
    w = _bf(n, k, seed=32, scale=0.02)
    sk = ops.StreamKBuffer(torch.empty(148 * 128 * 256, device="cuda"),
                           torch.zeros(1024 * 8, dtype=torch.int32, device="cuda"))
    ref = x.float() @ w.float().T
    outs = []
    for _ in range(3):
        out = torch.full((t, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        ops.linear(x, w, out=out, streamk=sk)
        outs.append(out)
    torch.testing.assert_close(outs[0].float(), ref, atol=2e-2, rtol=2e-2)
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    res = _bf(t, n, seed=33)
    out = res.clone()
    ops.linear(x, w, out=out, residual=out, streamk=sk)
    torch.testing.assert_close(out.float(), ref + res.float(), atol=3e-2, rtol=2e-2)
    assert int(sk.flags.abs().sum()) == 0
    assert ops.status("gemm_bf16") == 0


@pytest.mark.parametrize("t,n,k,bn", [(256, 28672, 4096, 256), (200, 19000, 1024, 128), (256, 128256, 4096, 256)])
def test_linear_streamk_wide_tiles(t, n, k, bn):
    """Stream-K with 128- and 256-token tiles (the TMA-store epilogue and a
    per-tile ticket), forced through a plan override: matches fp32 with and
    without the residual, bit-identical across launches, tickets reset."""
    import dataclasses

    from foundry_b200 import ops
    from foundry_b200.ops.gemm import plan

    p = dataclasses.replace(plan(t, n, k), bn=bn, splits=1, mt=1, grid=148, streamk=True, pair=False)
    x = _bf(t, k, seed=41)
    w = _bf(n, k, seed=42, scale=0.02)
    sk = ops.StreamKBuffer(torch.empty(148 * 128 * 256, device="cuda"),
                           torch.zeros(1024 * 8, dtype=torch.int32, device="cuda"))
    ref = x.float() @ w.float().T
    outs = []
    for _ in range(2):
        out = torch.full((t, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        ops.linear(x, w, out=out, streamk=sk, plan_override=p)
        outs.append(out)
    torch.testing.assert_close(outs[0].float(), ref, atol=2e-2, rtol=2e-2)
    assert torch.equal(outs[0], outs[1])
    res = _bf(t, n, seed=43)
    out = res.clone()
    ops.linear(x, w, out=out, residual=out, streamk=sk, plan_override=p)
    torch.testing.assert_close(out.float(), ref + res.float(), atol=3e-2, rtol=2e-2)
    assert int(sk.flags.abs().sum()) == 0
    assert ops.status("gemm_bf16") == 0


@pytest.mark.parametrize("t,inter,k,bn", [(256, 14336, 4096, None), (200, 1024, 512, None), (1, 1024, 512, None),
                                          (64, 3584, 8192, None), (256, 1024, 512, 256), (100, 1024, 512, 32),
                                          (130, 2048, 1024, 128), (40, 1024, 2048, 64)])
def test_linear_swiglu(t, inter, k, bn):
    """gate/up GEMM with the SiLU(gate) * up epilogue (two A tiles per unit:
    gate rows and the matching up rows) against fp32, for the planner's
    choice and forced tile widths."""
    import dataclasses

    from foundry_b200 import ops
    from foundry_b200.ops.gemm import plan_swiglu

    x = _bf(t, k, seed=51)
    w = _bf(2 * inter, k, seed=52, scale=0.05)
    p = plan_swiglu(t, inter, k)
    assert p is not None and p.mt == 2
    if bn is not None:
        p = dataclasses.replace(p, bn=bn, grid=min(148, (inter // 128) * -(-t // bn)))
    out = torch.full((t, inter), float("nan"), dtype=torch.bfloat16, device="cuda")
    assert ops.linear_swiglu(x, w, out, plan_override=p) is out
    gu = x.float() @ w.float().T
    ref = torch.nn.functional.silu(gu[:, :inter]) * gu[:, inter:]
    torch.testing.assert_close(out.float(), ref, atol=3e-2, rtol=2e-2)
    assert ops.status("gemm_bf16") == 0


@pytest.mark.parametrize("t,inter,k,pdl", [(256, 14336, 4096, True), (200, 11008, 4096, False),
                                           (160, 12288, 1024, True), (129, 9728, 2048, False)])
def test_linear_swiglu_streamk(t, inter, k, pdl):
    """Stream-K form of the fused gate/up + SwiGLU GEMM (every CTA an equal
    share of the (unit, k-block) iterations, units cut into up to three
    pieces summed by the last CTA) against fp32; a second launch gives the
    same bits (piece-order sums) and every launch leaves the flags zero."""
    import contextlib

    from foundry_b200 import ops
    from foundry_b200.ops import _rt
    from foundry_b200.ops.gemm import plan_swiglu_sk, swiglu_sk_sizes

    p = plan_swiglu_sk(t, inter, k, force=True)
    assert p is not None and p.streamk
    x = _bf(t, k, seed=61)
    w = _bf(2 * inter, k, seed=62, scale=0.05)
    ws_n, fl_n = swiglu_sk_sizes(inter)
    sk = ops.StreamKBuffer(torch.full((ws_n,), float("nan"), device="cuda"),
                           torch.zeros(fl_n, dtype=torch.int32, device="cuda"))
    out = torch.full((t, inter), float("nan"), dtype=torch.bfloat16, device="cuda")
    with _rt.pdl() if pdl else contextlib.nullcontext():
        assert ops.linear_swiglu(x, w, out, plan_override=p, sk=sk) is out
    first = out.clone()
    gu = x.float() @ w.float().T
    ref = torch.nn.functional.silu(gu[:, :inter]) * gu[:, inter:]
    torch.testing.assert_close(out.float(), ref, atol=3e-2, rtol=2e-2)
    assert int(sk.flags.abs().sum()) == 0
    out.fill_(float("nan"))
    with _rt.pdl() if pdl else contextlib.nullcontext():
        ops.linear_swiglu(x, w, out, plan_override=p, sk=sk)
    assert torch.equal(out, first)
    assert int(sk.flags.abs().sum()) == 0
    assert ops.status("gemm_bf16") == 0


@pytest.mark.parametrize("t,n,k", [(256, 4096, 4096), (256, 6144, 4096), (200, 4096, 1024), (64, 28672, 512)])
def test_linear_under_programmatic_dependent_launch(t, n, k):
    """Decode GEMMs launched with programmatic dependent launch (as inside
    the decode step: the weight tiles of the first ring are loaded before
    griddepcontrol.wait), back to back with kernels that write their inputs
    and outputs: same results as fp32, one-SM and two-SM plans, with and
    without split-K slices."""
    from foundry_b200 import ops
    from foundry_b200.ops import _rt

    w = _bf(n, k, seed=61, scale=0.02)
    ref_out = []
    outs = []
    pb = ops.PartialBuffer(8 * t * n)
    with _rt.pdl():
        for i in range(3):
            x0 = _bf(t, k, seed=70 + i)
            h = _bf(t, n, seed=80 + i)
            out = h.clone()
            ones = torch.ones(k, dtype=torch.bfloat16, device="cuda")
            x = torch.empty_like(x0)
            ops.rmsnorm(x0, ones, x, 1e-5)  # our kernel writes x right before the GEMMs read it
            ops.linear(x, w, out=out, residual=out)
            r = ops.linear(x, w, partials=pb)
            total = r.buf[: r.splits * r.stride].view(r.splits, t, n).sum(0) if isinstance(r, ops.Partial) else r.float()
            outs.append((out.float(), total.clone()))
            ref_out.append((h.float() + x.float() @ w.float().T, x.float() @ w.float().T))
    torch.cuda.synchronize()
    for (o, tot), (ro, rt) in zip(outs, ref_out):
        torch.testing.assert_close(o, ro, atol=4e-2, rtol=2e-2)
        torch.testing.assert_close(tot, rt, atol=4e-2, rtol=2e-2)
    assert ops.status("gemm_bf16") == 0
