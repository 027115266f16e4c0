"""GPU scenarios for the LD_PRELOAD interposer, each run in a fresh process
started by tests/test_interposer_gpu.py with libfoundry_hook.so preloaded
(the interposer must be in place before CUDA initialises).

    LD_PRELOAD=.../libfoundry_hook.so python tests/interposer_scenarios.py <name> <workdir>

Parity: reference tests/test_vmm_alloc.py, test_stop_resume.py,
test_preallocation.py, test_load_graph.py, test_load_cublas_ws.py (same
checks, our own scripts).
"""

from __future__ import annotations

import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

BASE = 0x500000000000
SIZE = 16 << 30


def _setup():
    import torch

    import foundry_b200 as fb

    assert fb.core().hook_is_preloaded(), "libfoundry_hook.so is not preloaded"
    torch.cuda.set_device(0)
    torch.cuda.init()
    return torch, fb


def scenario_region(workdir):
    torch, fb = _setup()
    fb.set_allocation_region(BASE, SIZE)
    ptrs = []
    keep = []
    for n in (1 << 10, 3 << 20, 64 << 20, 1 << 28, 5 << 20):
        t = torch.empty(n, dtype=torch.uint8, device="cuda")
        keep.append(t)
        ptrs.append(t.data_ptr())
    inside = [BASE <= p < BASE + SIZE for p in ptrs]
    assert all(inside), [hex(p) for p in ptrs]
    # segments come from a monotonically increasing cursor
    seg = sorted(set(p & ~((2 << 20) - 1) for p in ptrs))
    assert seg == sorted(seg)
    off = fb.get_current_alloc_offset()
    assert off > 0
    # stop: allocations bypass the region; resume: back inside
    fb.stop_allocation_region()
    torch.cuda.empty_cache()
    out = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    assert not (BASE <= out.data_ptr() < BASE + SIZE), hex(out.data_ptr())
    fb.resume_allocation_region()
    back = torch.empty(300 << 20, dtype=torch.uint8, device="cuda")
    assert BASE <= back.data_ptr() < BASE + SIZE
    # forward-only offset
    fb.set_current_alloc_offset(fb.get_current_alloc_offset() + (64 << 20))
    try:
        fb.set_current_alloc_offset(0)
        raise AssertionError("backwards offset accepted")
    except RuntimeError:
        pass
    x = torch.randn(1024, 1024, device="cuda")
    assert torch.isfinite((x @ x).sum())
    print(json.dumps({"ok": True, "ptrs": [hex(p) for p in ptrs], "intercepted": fb.core().intercepted_allocs()}))


def scenario_prealloc(workdir):
    torch, fb = _setup()
    import time

    fb.set_allocation_region(BASE, SIZE)
    assert fb.preallocate_region("4GB")
    t0 = time.perf_counter()
    ts = [torch.empty(n << 20, dtype=torch.uint8, device="cuda") for n in (2, 64, 512, 1024)]
    fast = time.perf_counter() - t0
    for t in ts:
        assert BASE <= t.data_ptr() < BASE + (4 << 30) + (64 << 20)
    ts[2].fill_(7)
    assert int(ts[2][12345]) == 7
    # past the window: slow path still lands in the region
    big = torch.empty(6 << 30, dtype=torch.uint8, device="cuda")
    assert BASE <= big.data_ptr() < BASE + SIZE
    print(json.dumps({"ok": True, "fast_path_s": fast}))


class _Net:
    def __init__(self, torch, seed=0):
        g = torch.Generator(device="cuda").manual_seed(seed)
        self.w1 = torch.randn(512, 256, device="cuda", generator=g) * 0.05
        self.b1 = torch.randn(512, device="cuda", generator=g) * 0.1
        self.w2 = torch.randn(128, 512, device="cuda", dtype=torch.float16, generator=g) * 0.05

    def __call__(self, torch, x):
        h = torch.nn.functional.gelu(x @ self.w1.T + self.b1)
        return (h.half() @ self.w2.T).float().softmax(-1)


def _prepare(torch, fb):
    fb.set_allocation_region(BASE, SIZE)
    fb.preallocate_cublas_workspaces()
    net = _Net(torch)
    static_x = torch.zeros(64, 256, device="cuda")
    # warm up every kernel outside capture (lazy module loads, cuBLAS heuristics)
    for _ in range(2):
        net(torch, static_x)
    torch.cuda.synchronize()
    return net, static_x


def scenario_graph_save(workdir):
    torch, fb = _setup()
    net, static_x = _prepare(torch, fb)
    g = fb.CUDAGraph()
    with fb.graph(g):
        y = net(torch, static_x)
    archive = os.path.join(workdir, "archive")
    os.makedirs(archive, exist_ok=True)
    g.save(os.path.join(archive, "graph_0.json"), output_tensors=y)
    fb.pack_fatbins_to_folder(archive)
    fb.save_graph_manifest(archive)
    x = torch.randn(64, 256, device="cuda", generator=torch.Generator(device="cuda").manual_seed(5))
    static_x.copy_(x)
    g.replay()
    torch.cuda.synchronize()
    ref = net(torch, x)
    torch.testing.assert_close(y, ref)
    torch.save(y.cpu(), os.path.join(workdir, "save_out.pt"))
    print(json.dumps({"ok": True, "nodes": g.desc.num_nodes, "kernels": g.desc.kernel_names()[:6],
                      "offset": fb.get_current_alloc_offset()}))


def scenario_graph_load(workdir):
    torch, fb = _setup()
    archive = os.path.join(workdir, "archive")
    fb.set_skip_fatbin_processing(True)
    fb.load_cuda_modules_and_libraries(archive)
    net, static_x = _prepare(torch, fb)
    g, y = fb.CUDAGraph.load(os.path.join(archive, "graph_0.json"))
    x = torch.randn(64, 256, device="cuda", generator=torch.Generator(device="cuda").manual_seed(5))
    static_x.copy_(x)
    g.replay()
    torch.cuda.synchronize()
    ref = net(torch, x)
    torch.testing.assert_close(y, ref)
    saved = torch.load(os.path.join(workdir, "save_out.pt"))
    assert torch.equal(y.cpu(), saved), "LOAD replay differs from SAVE replay"
    # a second input through the restored graph
    x2 = torch.randn(64, 256, device="cuda")
    static_x.copy_(x2)
    g.replay()
    torch.testing.assert_close(y, net(torch, x2))
    print(json.dumps({"ok": True}))


if __name__ == "__main__":
    name, workdir = sys.argv[1], sys.argv[2]
    {"region": scenario_region, "prealloc": scenario_prealloc, "graph_save": scenario_graph_save,
     "graph_load": scenario_graph_load}[name](workdir)
