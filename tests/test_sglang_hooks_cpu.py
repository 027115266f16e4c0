"""SGLang hooks (foundry_b200/integration/sglang/hooks.py) against a fake SGLang
package with the class and method names the hooks patch (SGLang is not
installed on this image), on the mock CUDA driver: install and uninstall,
workspace rank with and without DP attention, device binding + region +
scratch skip around init_torch_distributed, memory-pool config recorded in
SAVE and applied in LOAD, kernel warm-up skipped, warm-up forwards
suppressed, spawn sites exporting the preload and config."""

import os
import subprocess
import sys
import textwrap

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
MOCK = os.path.join(ROOT, "foundry_b200", "lib", "libfoundry_mockcuda.so")

FAKE = {
    "sglang/__init__.py": "",
    "sglang/srt/__init__.py": "",
    "sglang/srt/model_executor/__init__.py": "",
    "sglang/srt/model_executor/model_runner.py": """
        CALLS = []
        class ModelRunner:
            def init_torch_distributed(self):
                CALLS.append("init_torch_distributed")
                return "dist"
            def kernel_warmup(self):
                CALLS.append("kernel_warmup")
            def load_model(self):
                CALLS.append("load_model")
    """,
    "sglang/srt/model_executor/pool_configurator.py": """
        from dataclasses import dataclass
        @dataclass
        class MemoryPoolConfig:
            max_total_num_tokens: int = 0
            page_size: int = 1
    """,
    "sglang/srt/model_executor/model_runner_kv_cache_mixin.py": """
        from .pool_configurator import MemoryPoolConfig
        CALLS = []
        class ModelRunnerKVCacheMixin:
            def init_memory_pool(self, pre_model_load_memory):
                CALLS.append("init_memory_pool")
                self.memory_pool_config = MemoryPoolConfig(max_total_num_tokens=4242, page_size=16)
            def _apply_memory_pool_config(self, cfg):
                CALLS.append(("apply", cfg.max_total_num_tokens, cfg.page_size))
    """,
    "sglang/srt/model_executor/cuda_graph_runner.py": """
        _pool = None
        def get_global_graph_memory_pool():
            return _pool
        def set_global_graph_memory_pool(p):
            global _pool
            _pool = p
        class CudaGraphRunner:
            def capture(self):
                return "captured"
            def capture_one_batch_size(self, bs, forward, stream_idx=None):
                return None, None
            def _capture_graph(self, graph, pool, stream, run_once_fn):
                return run_once_fn()
            def _create_device_graph(self):
                return object()
    """,
    "sglang/srt/entrypoints/__init__.py": "",
    "sglang/srt/entrypoints/engine.py": """
        import os
        class Engine:
            def _launch_scheduler_processes(self):
                return (os.environ.get("LD_PRELOAD", ""), os.environ.get("FOUNDRY_GRAPH_CONFIG"),
                        os.environ.get("FOUNDRY_GRAPH_ENGINE"))
    """,
}

SCRIPT = r"""
import json, os, sys, types
sys.path.insert(0, FAKE_ROOT)
sys.path.insert(0, ROOT)
from foundry_b200 import get_current_alloc_offset
from foundry_b200.integration import runtime
from foundry_b200.integration.sglang import hooks as H
import sglang.srt.model_executor.model_runner as mr
import sglang.srt.model_executor.model_runner_kv_cache_mixin as kv
import sglang.srt.model_executor.cuda_graph_runner as cgr
import sglang.srt.entrypoints.engine as eng

# workspace rank: replicas stack after each other; with DP attention they are one TP world
sa = types.SimpleNamespace(tp_size=4, pp_size=2, dp_size=2, enable_dp_attention=False)
assert H.workspace_rank(sa, tp_rank=3, pp_rank=1, dp_rank=1) == 1 * 8 + 1 * 4 + 3
sa_dpa = types.SimpleNamespace(tp_size=4, pp_size=1, dp_size=4, enable_dp_attention=True)
assert H.workspace_rank(sa_dpa, tp_rank=2, pp_rank=0, dp_rank=3) == 2
assert H.sglang_graph_key(8, None) == 8 and H.sglang_graph_key(8, 1) == "1_8"
f = H.suppress_first_calls(lambda x: x * 2)
assert [f(1), f(2), f(3), f(4)] == [None, None, 6, 8]

orig = (mr.ModelRunner.init_torch_distributed, mr.ModelRunner.kernel_warmup, kv.ModelRunnerKVCacheMixin.init_memory_pool,
        cgr.CudaGraphRunner.capture, cgr.CudaGraphRunner.capture_one_batch_size, cgr.CudaGraphRunner._capture_graph,
        cgr.CudaGraphRunner._create_device_graph, eng.Engine._launch_scheduler_processes)
toml = os.path.join(TMP, MODE + ".toml")
with open(toml, "w") as fh:
    fh.write('mode = "%s"\nbase_addr = "0x620000000000"\nregion_size = "1GB"\nscratch_space_size = "32MB"\n'
             'workspace_root = "%s"\n' % (MODE, os.path.join(TMP, "arch")))
H.install_hooks(toml)
now = (mr.ModelRunner.init_torch_distributed, mr.ModelRunner.kernel_warmup, kv.ModelRunnerKVCacheMixin.init_memory_pool,
       cgr.CudaGraphRunner.capture, cgr.CudaGraphRunner.capture_one_batch_size, cgr.CudaGraphRunner._capture_graph,
       cgr.CudaGraphRunner._create_device_graph, eng.Engine._launch_scheduler_processes)
assert all(a is not b for a, b in zip(now, orig)) and H.installed()

# spawn site: the scheduler processes get the interposer and the config
pre, cfgp, engine = eng.Engine()._launch_scheduler_processes()
assert "libfoundry_hook.so" in pre and cfgp == toml and engine == "sglang", (pre, cfgp, engine)

class Runner(mr.ModelRunner, kv.ModelRunnerKVCacheMixin):
    pass
r = Runner()
r.device, r.gpu_id, r.tp_rank, r.pp_rank = "cpu", 0, 1, 0
r.server_args = types.SimpleNamespace(tp_size=2, pp_size=1, dp_size=1, enable_dp_attention=False)
assert r.init_torch_distributed() == "dist"
assert runtime.state().global_rank == 1 and get_current_alloc_offset() == 32 << 20
ws = os.path.join(TMP, "arch", "rank_1")
assert os.path.isdir(ws)
r.kernel_warmup()
assert "kernel_warmup" not in mr.CALLS
r.init_memory_pool(0)
state = json.load(open(os.path.join(ws, "warmup_state.json")))
if MODE == "save":
    assert kv.CALLS == ["init_memory_pool"], kv.CALLS
    assert state["extra"]["memory_pool_config"] == {"max_total_num_tokens": 4242, "page_size": 16}
else:
    assert kv.CALLS == [("apply", 4242, 16)], kv.CALLS
    assert r.memory_pool_config.max_total_num_tokens == 4242
g = cgr.CudaGraphRunner()
g.graphs, g.output_buffers = {}, {}
if MODE == "save":
    # after the capture loop: packed modules and the final offset are written
    assert g.capture() == "captured"
    for name in ("fatbin_entrypoint_packed.txt", "final_alloc_offset.json"):
        assert os.path.exists(os.path.join(ws, name)), name
else:
    cgr._pool = "pool"  # the engine's graph pool (a real one needs a device)
    assert g.capture() is None and g.graphs == {}  # LOAD replaces the capture loop (no graphs saved here)
H.uninstall_hooks()
assert (mr.ModelRunner.init_torch_distributed, mr.ModelRunner.kernel_warmup, kv.ModelRunnerKVCacheMixin.init_memory_pool,
        cgr.CudaGraphRunner.capture, cgr.CudaGraphRunner.capture_one_batch_size, cgr.CudaGraphRunner._capture_graph,
        cgr.CudaGraphRunner._create_device_graph, eng.Engine._launch_scheduler_processes) == orig
assert not H.installed() and runtime.state() is None
print("SGLANG_OK", MODE)
"""


def _fake_tree(root):
    for rel, src in FAKE.items():
        p = root / rel
        p.parent.mkdir(parents=True, exist_ok=True)
        p.write_text(textwrap.dedent(src))


def test_sglang_hooks_save_then_load_on_fake_sglang(tmp_path):
    fake = tmp_path / "fake"
    _fake_tree(fake)
    env = dict(os.environ, FOUNDRY_CUDA_DRIVER=MOCK, PYTHONPATH=ROOT, CUDA_VISIBLE_DEVICES="")
    env.pop("LD_PRELOAD", None)
    for mode in ("save", "load"):
        code = f"ROOT={ROOT!r}; TMP={str(tmp_path)!r}; FAKE_ROOT={str(fake)!r}; MODE={mode!r}\n" + SCRIPT
        r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=180)
        assert r.returncode == 0 and f"SGLANG_OK {mode}" in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]


def test_missing_required_target_patches_nothing(tmp_path):
    fake = tmp_path / "fake"
    _fake_tree(fake)
    # an SGLang without CudaGraphRunner.capture_one_batch_size: install must fail before patching anything
    cgr = fake / "sglang/srt/model_executor/cuda_graph_runner.py"
    cgr.write_text(cgr.read_text().replace("def capture_one_batch_size", "def other_name"))
    code = textwrap.dedent(f"""
        import sys
        sys.path.insert(0, {str(fake)!r}); sys.path.insert(0, {ROOT!r})
        from foundry_b200.integration.sglang import hooks as H
        from foundry_b200.integration.config import GraphExtensionConfig
        import sglang.srt.model_executor.model_runner as mr
        before = mr.ModelRunner.init_torch_distributed
        try:
            H.install_hooks(GraphExtensionConfig.from_dict({{"mode": "save"}}))
            raise SystemExit("installed on an unsupported SGLang")
        except ImportError as e:
            assert "capture_one_batch_size" in str(e), e
        assert mr.ModelRunner.init_torch_distributed is before and not H.installed()
        print("MISSING_OK")
    """)
    env = dict(os.environ, PYTHONPATH=ROOT, CUDA_VISIBLE_DEVICES="", FOUNDRY_CUDA_DRIVER=MOCK)
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=180)
    assert r.returncode == 0 and "MISSING_OK" in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]


def test_serve_launcher_environment(tmp_path):
    """The SGLang launcher preloads the interposer, exports the config and the
    engine selector, puts the shim first on PYTHONPATH and turns NCCL's cuMem
    and NVLS paths off; the recipes parse."""
    from foundry_b200.integration.config import GraphExtensionConfig, GraphExtensionMode
    from foundry_b200.integration.sglang.serve import build_command

    recipes = os.path.join(ROOT, "foundry_b200", "integration", "sglang", "recipes")
    toml = os.path.join(recipes, "foundry_save.toml")
    assert GraphExtensionConfig.from_toml(toml).mode == GraphExtensionMode.SAVE
    assert GraphExtensionConfig.from_toml(os.path.join(recipes, "foundry_load.toml")).mode == GraphExtensionMode.LOAD
    cmd, env = build_command(["--foundry-config", toml, "--", "--model-path", "m", "--tp-size", "2"],
                             environ={"PYTHONPATH": "/x", "NCCL_NVLS_ENABLE": "1"})
    assert cmd[1:3] == ["-m", "sglang.launch_server"] and cmd[3:] == ["--model-path", "m", "--tp-size", "2"]
    assert env["FOUNDRY_GRAPH_ENGINE"] == "sglang" and env["FOUNDRY_GRAPH_CONFIG"] == os.path.abspath(toml)
    assert env["PYTHONPATH"].split(os.pathsep)[0].endswith(os.path.join("vllm", "_site"))
    assert env["PYTHONPATH"].split(os.pathsep)[-1] == "/x"
    assert env["NCCL_CUMEM_ENABLE"] == "0" and env["NCCL_NVLS_ENABLE"] == "1"  # explicit settings win
    assert "libfoundry_hook.so" in env.get("LD_PRELOAD", "")
