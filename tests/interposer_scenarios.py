"""GPU scenarios for the LD_PRELOAD interposer, each run in a fresh process
started by tests/test_interposer_gpu.py with libfoundry_hook.so preloaded
(the interposer must be in place before CUDA initialises).

    LD_PRELOAD=.../libfoundry_hook.so python tests/interposer_scenarios.py <name> <workdir>

Parity: reference tests/test_vmm_alloc.py, test_stop_resume.py,
test_preallocation.py, test_load_graph.py, test_load_cublas_ws.py,
test_async_load.py (same checks, our own scripts).
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


# ---- many graphs, shared topologies, asynchronous restore ---------------------------------
ASYNC_SIZES = [8, 16, 32, 64, 128, 256, 8, 16, 512, 1024, 32, 64]


class _Mlp:
    """4 layers of fp16 GEMM + bias + SiLU (cuBLAS + libtorch elementwise kernels)."""

    def __init__(self, torch, width=384, layers=4):
        g = torch.Generator(device="cuda").manual_seed(7)
        self.ws = [(torch.randn(width, width, device="cuda", generator=g) * 0.05).half() for _ in range(layers)]
        self.bs = [(torch.randn(width, device="cuda", generator=g) * 0.1).half() for _ in range(layers)]

    def __call__(self, torch, x):
        for w, b in zip(self.ws, self.bs):
            x = torch.nn.functional.silu(torch.addmm(b, x, w.T))
        return x


def _async_prepare(torch, fb):
    """Weights, every static input and the warm-up, all before any capture,
    in the same order in SAVE and LOAD (the region cursor must agree)."""
    fb.set_allocation_region(BASE, SIZE)
    fb.preallocate_cublas_workspaces()
    net = _Mlp(torch)
    xs = [torch.zeros(bs, 384, device="cuda", dtype=torch.float16) for bs in ASYNC_SIZES]
    for _ in range(2):
        for x in xs:
            net(torch, x)
    torch.cuda.synchronize()
    return net, xs


def _async_inputs(torch, i):
    g = torch.Generator(device="cuda").manual_seed(100 + i)
    return torch.randn(ASYNC_SIZES[i], 384, device="cuda", generator=g).half()


def scenario_async_save(workdir):
    torch, fb = _setup()
    net, xs = _async_prepare(torch, fb)
    archive = os.path.join(workdir, "archive")
    os.makedirs(archive, exist_ok=True)
    pool = fb.graph_pool_handle()
    graphs, outs = [], []
    for x in xs:
        g = fb.CUDAGraph()
        with fb.graph(g, pool=pool):
            y = net(torch, x)
        graphs.append(g)
        outs.append(y)
    for i, (g, y) in enumerate(zip(graphs, outs)):
        g.save(os.path.join(archive, f"graph_{i}.json"), output_tensors=y)
    fb.pack_fatbins_to_folder(archive)
    manifest = fb.save_graph_manifest(archive)
    results = []
    for i, (g, x, y) in enumerate(zip(graphs, xs, outs)):
        x.copy_(_async_inputs(torch, i))
        g.replay()
        torch.cuda.synchronize()
        torch.testing.assert_close(y, net(torch, x), rtol=2e-3, atol=2e-3)
        results.append(y.cpu().clone())
    torch.save(results, os.path.join(workdir, "async_out.pt"))
    groups = len(manifest["topology_groups"]) if manifest else len(ASYNC_SIZES)
    print(json.dumps({"ok": True, "graphs": len(graphs), "groups": groups}))


def scenario_async_load(workdir):
    import time

    torch, fb = _setup()
    archive = os.path.join(workdir, "archive")
    fb.set_skip_fatbin_processing(True)
    fb.load_cuda_modules_and_libraries(archive)
    net, xs = _async_prepare(torch, fb)
    paths = [os.path.join(archive, f"graph_{i}.json") for i in range(len(ASYNC_SIZES))]
    t0 = time.perf_counter()
    pending = fb.CUDAGraph.start_graph_builds(paths)
    started = time.perf_counter() - t0
    busy = sum(i * i for i in range(200_000))  # host work overlapping the background builds
    loaded = fb.CUDAGraph.finish_graph_loads(pending)
    total = time.perf_counter() - t0
    saved = torch.load(os.path.join(workdir, "async_out.pt"))
    # replay in an order unlike capture order: on-demand members patch their template
    for i in [3, 0, 7, 1, 11, 6, 2, 9, 4, 8, 10, 5]:
        g, y = loaded[i]
        xs[i].copy_(_async_inputs(torch, i))
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(y.cpu(), saved[i]), f"graph {i}: LOAD replay differs from SAVE replay"
        torch.testing.assert_close(y, net(torch, xs[i]), rtol=2e-3, atol=2e-3)
    print(json.dumps({"ok": busy > 0, "start_s": started, "restore_s": total}))


# ---- random numbers inside a persisted graph -------------------------------------------
RNG_N = 1 << 16


def _rng_prepare(torch, fb):
    """Same allocations in SAVE and LOAD, before any capture."""
    fb.set_allocation_region(BASE, SIZE)
    x = torch.zeros(RNG_N, device="cuda")
    for _ in range(2):  # load the RNG kernels outside capture
        _rng_body(torch, x)
    torch.cuda.synchronize()
    return x


def _rng_body(torch, x):
    return x + torch.rand_like(x) + torch.nn.functional.dropout(torch.ones_like(x), p=0.5)


def scenario_rng_save(workdir):
    torch, fb = _setup()
    x = _rng_prepare(torch, fb)
    g = fb.CUDAGraph()
    with fb.graph(g):
        y = _rng_body(torch, x)
    gens = g.desc.generators
    assert len(gens) == 1 and gens[0]["wholegraph_increment"] > 0 and gens[0]["seed_ptr"], gens
    archive = os.path.join(workdir, "archive")
    os.makedirs(archive, exist_ok=True)
    g.save(os.path.join(archive, "graph_0.json"), output_tensors=y)
    fb.pack_fatbins_to_folder(archive)
    fb.save_graph_manifest(archive)
    torch.cuda.manual_seed(1234)
    gen = torch.cuda.default_generators[0]
    off0 = gen.get_offset()
    outs = []
    for i in range(3):
        x.fill_(float(i))
        g.replay()
        outs.append(y.cpu().clone())
    inc = gens[0]["wholegraph_increment"]
    # the recorded increment is the one torch's replay applies
    assert gen.get_offset() - off0 == 3 * inc, (gen.get_offset(), off0, inc)
    assert not torch.equal(outs[0], outs[1] - 1), "replays drew the same random numbers"
    torch.save(outs, os.path.join(workdir, "rng_out.pt"))
    print(json.dumps({"ok": True, "increment": inc}))


def scenario_rng_load(workdir):
    torch, fb = _setup()
    archive = os.path.join(workdir, "archive")
    fb.set_skip_fatbin_processing(True)
    fb.load_cuda_modules_and_libraries(archive)
    x = _rng_prepare(torch, fb)
    g, y = fb.CUDAGraph.load(os.path.join(archive, "graph_0.json"))
    saved = torch.load(os.path.join(workdir, "rng_out.pt"))
    torch.cuda.manual_seed(1234)
    for i in range(3):
        x.fill_(float(i))
        g.replay()
        assert torch.equal(y.cpu(), saved[i]), f"replay {i}: restored graph drew other random numbers"
    # another seed gives another sequence
    torch.cuda.manual_seed(99)
    x.fill_(0.0)
    g.replay()
    assert not torch.equal(y.cpu(), saved[0])
    print(json.dumps({"ok": True}))


# ---- torch.compile (Inductor / Triton) kernels in a persisted graph -------------------------
def _compile_inputs(torch):
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn(1 << 16, device="cuda", generator=g)
    y = torch.randn(1 << 16, device="cuda", generator=g)
    return x, y


def _eager(torch, x, y):
    return torch.sin(x * 1.5 + y) * y - torch.relu(x)


def scenario_compile_save(workdir):
    torch, fb = _setup()
    from foundry_b200 import jit

    fb.set_allocation_region(BASE, SIZE)
    x, y = _compile_inputs(torch)
    fn = torch.compile(lambda a, b: _eager(torch, a, b), dynamic=False)
    for _ in range(3):  # compile + warm-up: Triton loads (and foundry adopts) the kernel here
        fn(x, y)
    torch.cuda.synchronize()
    assert jit.installed() and jit.adopted, "no Triton kernel was adopted"
    g = fb.CUDAGraph()
    with fb.graph(g):
        z = fn(x, y)
    names = g.desc.kernel_names()
    assert any("triton" in n for n in names), names
    archive = os.path.join(workdir, "archive")
    os.makedirs(archive, exist_ok=True)
    g.save(os.path.join(archive, "graph_0.json"), output_tensors=z)
    fb.pack_fatbins_to_folder(archive)
    fb.save_graph_manifest(archive)
    g.replay()
    torch.cuda.synchronize()
    torch.testing.assert_close(z, _eager(torch, x, y), rtol=1e-5, atol=1e-5)
    torch.save(z.cpu(), os.path.join(workdir, "compile_out.pt"))
    print(json.dumps({"ok": True, "kernels": names, "adopted": len(jit.adopted)}))


def scenario_compile_load(workdir):
    torch, fb = _setup()
    archive = os.path.join(workdir, "archive")
    fb.set_skip_fatbin_processing(True)
    fb.load_cuda_modules_and_libraries(archive)
    fb.set_allocation_region(BASE, SIZE)
    x, y = _compile_inputs(torch)
    g, z = fb.CUDAGraph.load(os.path.join(archive, "graph_0.json"))
    g.replay()
    torch.cuda.synchronize()
    saved = torch.load(os.path.join(workdir, "compile_out.pt"))
    assert torch.equal(z.cpu(), saved), "restored torch.compile graph differs from SAVE"
    x.mul_(0.5)
    g.replay()
    torch.testing.assert_close(z, _eager(torch, x, y), rtol=1e-5, atol=1e-5)
    # nothing was compiled in this process
    assert "torch._inductor.compile_fx" not in sys.modules
    print(json.dumps({"ok": True}))


if __name__ == "__main__":
    name, workdir = sys.argv[1], sys.argv[2]
    {"region": scenario_region, "prealloc": scenario_prealloc, "graph_save": scenario_graph_save,
     "graph_load": scenario_graph_load, "async_save": scenario_async_save,
     "async_load": scenario_async_load, "rng_save": scenario_rng_save,
     "rng_load": scenario_rng_load, "compile_save": scenario_compile_save,
     "compile_load": scenario_compile_load}[name](workdir)
