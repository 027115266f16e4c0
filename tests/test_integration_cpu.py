"""Engine integrations on CPU: TOML config, archive file naming, the region
setup / scratch skip / final-offset check on the mock driver, and the vLLM
hooks being installable and removable against the installed vLLM."""

import os
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
MOCK = os.path.join(ROOT, "foundry_b200", "lib", "libfoundry_mockcuda.so")


def test_config_from_toml(tmp_path):
    from foundry_b200.integration.config import GraphExtensionConfig, GraphExtensionMode, global_rank

    p = tmp_path / "c.toml"
    p.write_text('mode = "save"\nbase_addr = "0x610000000000"\nregion_size = "8GB"\n'
                 'workspace_root = "arch"\nscratch_space_size = "32MB"\n')
    c = GraphExtensionConfig.from_toml(p)
    assert c.mode == GraphExtensionMode.SAVE and c.base_addr == 0x610000000000
    assert c.workspace_for(global_rank(1, 2, dp_rank=1)) == os.path.join("arch", "rank_3")
    assert GraphExtensionConfig.from_dict({}).mode == GraphExtensionMode.NONE
    with pytest.raises(ValueError):
        GraphExtensionConfig.from_dict({"mode": "save", "bogus": 1})
    with pytest.raises(ValueError):
        GraphExtensionConfig.from_dict({"mode": "frobnicate"})
    with pytest.raises(ValueError):
        GraphExtensionConfig.from_dict({"region_size": "1GB", "scratch_space_size": "2GB"})
    recipes = os.path.join(ROOT, "foundry_b200", "integration", "vllm", "recipes")
    assert GraphExtensionConfig.from_toml(os.path.join(recipes, "foundry_load.toml")).mode == GraphExtensionMode.LOAD


def test_graph_filename_codec():
    from foundry_b200.integration.graph_ops import GraphKey, parse_filename

    keys = [GraphKey("FULL", 256, 256, True, False, None), GraphKey("PIECEWISE", 8, None, False, True, 3),
            GraphKey("FULL_DECODE_ONLY", 1, 1, True, False, None)]
    for i, k in enumerate(keys):
        name = k.filename(i)
        assert parse_filename(name) == (i, k)
    assert keys[0].filename(7) == "graph_7_FULL_t256_r256_UX_pcN.json"
    assert parse_filename("graph_manifest.json") is None


RUNTIME = r"""
import json, os, sys
sys.path.insert(0, ROOT)
from foundry_b200 import core, get_current_alloc_offset
from foundry_b200.integration import runtime
from foundry_b200.integration.config import GraphExtensionConfig
ws = os.path.join(TMP, "arch")
cfg = GraphExtensionConfig.from_dict({"mode": "save", "region_size": "1GB", "scratch_space_size": "64MB",
                                      "workspace_root": ws, "base_addr": "0x600000000000"})
runtime.setup_graph_extension(cfg, 0)
assert runtime.skip_to_scratch_boundary() == 64 << 20
assert get_current_alloc_offset() == 64 << 20
p = core().region_alloc(4 << 20)
assert p >= 0x600000000000 + (64 << 20)
sizes = [3 << 20, 64 << 20, 5 << 20, 300 << 20, 2 << 20]
addrs = [core().region_alloc(n) for n in sizes]
off = runtime.capture_final_alloc_offset()
assert json.load(open(os.path.join(ws, "rank_0", "final_alloc_offset.json")))["final_alloc_offset"] == off
from foundry_b200 import pack_fatbins_to_folder
pack_fatbins_to_folder(os.path.join(ws, "rank_0"))
json.dump({"first": p, "addrs": addrs}, open(os.path.join(TMP, "save_addrs.json"), "w"))
env = runtime.ld_preload_env({"LD_PRELOAD": "/x.so"})
assert env["LD_PRELOAD"].split(":")[-1] == "/x.so" and "libfoundry_hook.so" in env["LD_PRELOAD"]
print("RUNTIME_OK")
"""

RUNTIME_LOAD = r"""
import json, os, sys
sys.path.insert(0, ROOT)
from foundry_b200 import core
from foundry_b200.integration import graph_ops, runtime
from foundry_b200.integration.config import GraphExtensionConfig
ws = os.path.join(TMP, "arch")
cfg = GraphExtensionConfig.from_dict({"mode": "load", "region_size": "1GB", "scratch_space_size": "64MB",
                                      "workspace_root": ws, "base_addr": "0x600000000000"})
runtime.setup_graph_extension(cfg, 0)
runtime.skip_to_scratch_boundary()
want = json.load(open(os.path.join(TMP, "save_addrs.json")))
mapped = runtime.preallocate_for_load_mode()
final = json.load(open(os.path.join(ws, "rank_0", "final_alloc_offset.json")))["final_alloc_offset"]
assert mapped == final - (64 << 20), (mapped, final)
got = [core().region_alloc(4 << 20)] + [core().region_alloc(n) for n in [3 << 20, 64 << 20, 5 << 20, 300 << 20, 2 << 20]]
assert got == [want["first"]] + want["addrs"], (got, want)
runtime.capture_final_alloc_offset()  # raises if the cursor drifted from SAVE's
plan = graph_ops.start_graph_builds(cfg.workspace_dir)
assert graph_ops.start_graph_builds(cfg.workspace_dir) is plan and plan.paths == []
print("RUNTIME_LOAD_OK")
"""


def test_runtime_region_scratch_and_final_offset_on_mock(tmp_path):
    env = dict(os.environ, FOUNDRY_CUDA_DRIVER=MOCK, PYTHONPATH=ROOT, CUDA_VISIBLE_DEVICES="")
    code = f"ROOT={ROOT!r}; TMP={str(tmp_path)!r}\n" + RUNTIME
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=180)
    assert r.returncode == 0 and "RUNTIME_OK" in r.stdout, r.stdout + r.stderr[-3000:]
    # LOAD: one preallocated window up to SAVE's final offset gives the same addresses
    code = f"ROOT={ROOT!r}; TMP={str(tmp_path)!r}\n" + RUNTIME_LOAD
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=180)
    assert r.returncode == 0 and "RUNTIME_LOAD_OK" in r.stdout, r.stdout + r.stderr[-3000:]


VLLM_HOOKS = r"""
import sys
sys.path.insert(0, ROOT)
import vllm.compilation.cuda_graph as cg
import vllm.v1.worker.gpu_worker as gw
import vllm.v1.worker.gpu_model_runner as mr
import types, torch
from vllm.config import CUDAGraphMode
R = mr.GPUModelRunner
orig = (cg.CUDAGraphWrapper.__call__, gw.init_worker_distributed_environment, gw.kernel_warmup, R.capture_model,
        R.load_model, R._dummy_run, R.initialize_kv_cache, torch.cuda.get_device_capability)
from foundry_b200.integration import runtime
from foundry_b200.integration.vllm import install_hooks, installed, uninstall_hooks
from foundry_b200.integration.vllm.hooks import is_sampler_warmup_run
from foundry_b200.integration.config import GraphExtensionConfig
cfg = GraphExtensionConfig.from_dict({"mode": "save"})
install_hooks(cfg)
assert installed()
now = (cg.CUDAGraphWrapper.__call__, gw.init_worker_distributed_environment, gw.kernel_warmup, R.capture_model,
       R.load_model, R._dummy_run, R.initialize_kv_cache, torch.cuda.get_device_capability)
assert all(a is not b for a, b in zip(now, orig)), now
# only the eager sampler warm-up forward is replaced
none = CUDAGraphMode.NONE
assert is_sampler_warmup_run({"cudagraph_runtime_mode": none, "skip_eplb": True})
for extra in ("is_profile", "is_graph_capturing", "force_attention", "uniform_decode"):
    assert not is_sampler_warmup_run({"cudagraph_runtime_mode": none, "skip_eplb": True, extra: True})
assert not is_sampler_warmup_run({"skip_eplb": True})
assert not is_sampler_warmup_run({"cudagraph_runtime_mode": CUDAGraphMode.FULL, "skip_eplb": True})
runtime._state = runtime.ExtensionState(cfg, 0)
fake = types.SimpleNamespace(model_config=types.SimpleNamespace(get_hidden_size=lambda: 16, dtype=torch.float32),
                             device="cpu")
hs, last = R._dummy_run(fake, 4, cudagraph_runtime_mode=none, skip_eplb=True)
assert hs.shape == (4, 16) and not hs.any() and last is hs
uninstall_hooks()
assert (cg.CUDAGraphWrapper.__call__, gw.init_worker_distributed_environment, gw.kernel_warmup, R.capture_model,
        R.load_model, R._dummy_run, R.initialize_kv_cache, torch.cuda.get_device_capability) == orig
print("HOOKS_OK")
"""


def test_nvml_capability_without_cuda_context():
    from foundry_b200.integration.vllm.hooks import nvml_device_capability

    class FakeNvml:
        def __init__(self):
            self.inits, self.asked = 0, []

        def nvmlInit(self):
            self.inits += 1

        def nvmlDeviceGetHandleByIndex(self, i):
            self.asked.append(i)
            return ("h", i)

        def nvmlDeviceGetCudaComputeCapability(self, h):
            return (10, 0) if h[1] == 0 else (9, 0)

    nv = FakeNvml()
    assert nvml_device_capability(None, _nvml=nv) == (10, 0)
    assert nvml_device_capability(1, _nvml=nv) == (9, 0)
    assert nvml_device_capability("cuda:1", _nvml=nv) == (9, 0)
    import torch

    assert nvml_device_capability(torch.device("cuda", 0), _nvml=nv) == (10, 0)
    assert nv.inits == 1 and nv.asked == [0, 1, 1, 0]


def test_vllm_hooks_install_and_uninstall():
    pytest.importorskip("vllm")
    env = dict(os.environ, PYTHONPATH=ROOT, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([sys.executable, "-c", f"ROOT={ROOT!r}\n" + VLLM_HOOKS], env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0 and "HOOKS_OK" in r.stdout, r.stdout[-2000:] + r.stderr[-3000:]


def test_materialize_loaded_graphs_in_background():
    """LOAD: every restored graph gets its own executable, largest first, on a
    background thread (fake graphs record the order)."""
    from foundry_b200.integration import graph_ops, runtime
    from foundry_b200.integration.config import GraphExtensionConfig

    order = []

    class FakeGraph:
        def __init__(self, n):
            self.n = n

        def materialize(self):
            order.append(self.n)

    st = runtime.ExtensionState(GraphExtensionConfig.from_dict({"mode": "load"}), 0)
    for n in (8, 256, 1, 64):
        st.loaded[graph_ops.GraphKey("FULL", n, n, True, False, None)] = (FakeGraph(n), None)
    runtime._state = st
    try:
        t = graph_ops.materialize_loaded(background=True)
        t.join(timeout=30)
        assert order == [256, 64, 8, 1]
        runtime._state = runtime.ExtensionState(GraphExtensionConfig.from_dict({"mode": "load"}), 0)
        assert graph_ops.materialize_loaded() is None  # nothing restored yet
    finally:
        runtime.reset()


def test_vllm_serve_launcher_environment():
    """The vLLM launcher preloads the interposer, exports the config, puts the
    shim first on PYTHONPATH and turns NCCL's cuMem and NVLS paths off."""
    from foundry_b200.integration.vllm.serve import build_command

    toml = os.path.join(ROOT, "foundry_b200", "integration", "vllm", "recipes", "foundry_load.toml")
    cmd, env = build_command(["--foundry-config", toml, "--", "Qwen/Qwen3-30B-A3B-FP8", "--data-parallel-size", "2"],
                             environ={})
    assert "serve" in cmd and cmd[-3:] == ["Qwen/Qwen3-30B-A3B-FP8", "--data-parallel-size", "2"]
    assert env["FOUNDRY_GRAPH_CONFIG"] == os.path.abspath(toml) and "FOUNDRY_SPAWN_T0_NS" in env
    assert env["PYTHONPATH"].split(os.pathsep)[0].endswith(os.path.join("vllm", "_site"))
    assert env["NCCL_CUMEM_ENABLE"] == "0" and env["NCCL_NVLS_ENABLE"] == "0"
    assert "libfoundry_hook.so" in env.get("LD_PRELOAD", "")


def test_vllm_deepep_and_nvshmem_flush_patches():
    """The DeepEP kwargs patch forces fabric buffers whenever graphs are
    persisted; the communication-buffer patch initialises NVSHMEM images on
    LOAD only, after the original ran."""
    import types

    from foundry_b200.integration import runtime
    from foundry_b200.integration.config import GraphExtensionConfig
    from foundry_b200.integration.vllm import hooks

    saved = dict(hooks._originals)
    calls = []
    try:
        hooks._originals["DeepEPLLAll2AllManager._make_all2all_kwargs"] = lambda self: {"use_fabric": False,
                                                                                          "num_nvl_bytes": 1 << 30}
        hooks._originals["prepare_communication_buffer_for_model"] = lambda model: calls.append(("orig", model))
        runtime._state = runtime.ExtensionState(GraphExtensionConfig.from_dict({"mode": "save"}), 0)
        assert hooks._deepep_kwargs(object()) == {"use_fabric": True, "num_nvl_bytes": 0}
        hooks._prepare_comm_buffer("m")
        assert calls == [("orig", "m")]  # SAVE: no NVSHMEM init
        runtime._state = runtime.ExtensionState(GraphExtensionConfig.from_dict({"mode": "none"}), 0)
        assert hooks._deepep_kwargs(object())["use_fabric"] is False
        runtime._state = runtime.ExtensionState(GraphExtensionConfig.from_dict({"mode": "load"}), 0)
        import foundry_b200

        orig_init = foundry_b200.init_nvshmem_for_loaded_modules
        foundry_b200.init_nvshmem_for_loaded_modules = lambda: calls.append("nvshmem") or 3
        try:
            hooks._prepare_comm_buffer("m2")
        finally:
            foundry_b200.init_nvshmem_for_loaded_modules = orig_init
        assert calls[-2:] == [("orig", "m2"), "nvshmem"]
    finally:
        hooks._originals.clear()
        hooks._originals.update(saved)
        runtime.reset()
