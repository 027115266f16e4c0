"""The allocation-free decode-attention entry point (lib/libfoundry_noalloc.so,
exported C symbol fb_decode_attention_noalloc, declared in
csrc/noalloc/decode_attn_noalloc.h) against the cubin entry point
(ops.decode_attention, impl="simt", same kernels with a caller-owned
workspace), on two calls in a row; the second call must leave the device's
free memory and torch's allocator untouched. Plus its size and argument
rejections. Named to be collected last; it must also pass alone in a fresh
process."""

import ctypes
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "foundry_b200", "lib",
                   "libfoundry_noalloc.so")
HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "csrc", "noalloc",
                      "decode_attn_noalloc.h")
MAX_PARTIAL_ROWS = 16384


def _entry():
    if not os.path.exists(LIB):
        raise RuntimeError(f"{LIB} is missing: run python -m foundry_b200._build")
    fn = ctypes.CDLL(LIB).fb_decode_attention_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int]
    return fn


def _case(batch, n_q, n_kv, max_pages, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    blocks = batch * max_pages + 3
    q = torch.randn(batch, n_q, 128, device="cuda", generator=g).to(torch.bfloat16)
    kc = torch.randn(blocks, n_kv, 64, 128, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(blocks, n_kv, 64, 128, device="cuda", generator=g).to(torch.bfloat16)
    perm = torch.randperm(blocks, device="cuda", generator=g)[: batch * max_pages]
    tables = perm.view(batch, max_pages).to(torch.int32).contiguous()
    lens = torch.randint(1, max_pages * 64 + 1, (batch,), device="cuda", generator=g).to(torch.int32)
    lens[0] = 1
    lens[-1] = max_pages * 64
    return q, kc, vc, tables, lens


def _call(fn, q, kc, vc, tables, lens, out, splits, pps, scale):
    err = ctypes.create_string_buffer(256)
    b, n_q, _ = q.shape
    rc = fn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), tables.data_ptr(), tables.shape[1], lens.data_ptr(),
            out.data_ptr(), b, n_q, kc.shape[1], splits, pps, scale, torch.cuda.current_stream().cuda_stream,
            err, len(err))
    return rc, err.value.decode()


@pytest.mark.parametrize("batch,n_q,n_kv,max_pages,splits", [(8, 32, 8, 10, 5), (3, 64, 8, 6, 3), (5, 32, 8, 4, 1)])
def test_no_alloc_matches_workspace_entry_point(batch, n_q, n_kv, max_pages, splits):
    from foundry_b200 import ops
    from foundry_b200.ops.attention import DecodeWorkspace

    fn = _entry()
    q, kc, vc, tables, lens = _case(batch, n_q, n_kv, max_pages, seed=batch * 100 + n_q)
    pps = -(-max_pages // splits)
    scale = 1.0 / 128 ** 0.5
    ws = DecodeWorkspace(batch, n_q, splits)
    want = torch.empty_like(q)
    ops.decode_attention(q, kc, vc, tables, lens, want, max_pages, ws, scale=scale, splits=(splits, pps),
                         impl="simt")
    assert ops.status("attention") == 0
    for call in range(2):  # the first call does the per-context setup; the second reuses it
        out = torch.full_like(q, float("nan"))
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        torch_before = torch.cuda.memory_allocated()
        rc, msg = _call(fn, q, kc, vc, tables, lens, out, splits, pps, scale)
        assert rc == 0, msg
        torch.cuda.synchronize()
        if call == 1:
            assert torch.cuda.mem_get_info()[0] == free_before, "the entry point allocated device memory"
            assert torch.cuda.memory_allocated() == torch_before
        torch.testing.assert_close(out.float(), want.float(), atol=2e-2, rtol=2e-2)


def test_no_alloc_header_declares_the_entry_point():
    text = open(HEADER).read()
    assert "int fb_decode_attention_noalloc(" in text
    assert f"#define FB_NOALLOC_MAX_PARTIAL_ROWS {MAX_PARTIAL_ROWS}" in text


def test_no_alloc_rejects_oversize_and_bad_args():
    fn = _entry()
    q, kc, vc, tables, lens = _case(8, 32, 8, 4, seed=3)
    out = torch.empty_like(q)
    # 8 * 32 * 65 partial rows > 16384: refused before any launch
    rc, msg = _call(fn, q, kc, vc, tables, lens, out, 65, 1, 0.1)
    assert rc == 1 and "scratch" in msg, msg
    assert 8 * 32 * 65 > MAX_PARTIAL_ROWS
    # GQA group 3 is not supported
    rc, msg = _call(fn, q[:, :24].contiguous(), kc, vc, tables, lens, out, 2, 2, 0.1)
    assert rc == 2 and "GQA" in msg, msg
    # splits * pages_per_split must cover the block table
    rc, msg = _call(fn, q, kc, vc, tables, lens, out, 1, 2, 0.1)
    assert rc == 2 and "cover" in msg, msg
