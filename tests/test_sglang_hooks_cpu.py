"""SGLang hooks (foundry_b200/integration/sglang/hooks.py) against a fake SGLang
package with the class and method names the hooks patch (SGLang is not
installed on this image), on the mock CUDA driver: install and uninstall,
workspace rank with and without DP attention, device binding + region +
scratch skip around init_torch_distributed, memory-pool config recorded in
SAVE and applied in LOAD, kernel warm-up skipped, warm-up forwards
suppressed, spawn sites exporting the preload and config, the FlashInfer
per-batch-size metadata pre-pass and the DeepEP buffer bootstrap."""

import os
import subprocess
import sys
import textwrap

import pytest

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


# A fake SGLang whose capture loop builds attention metadata per batch size the
# way SGLang's FlashInfer backend does (a new wrapper object per call), and
# whose MoE backend can be DeepEP: the pre-pass and the DeepEP bootstrap of
# foundry_b200/integration/sglang/prepass.py against it.
PREPASS_FAKE = {
    "sglang/srt/layers/__init__.py": "",
    "sglang/srt/layers/attention/__init__.py": "",
    "sglang/srt/layers/attention/flashinfer_backend.py": """
        EVENTS = []
        class DecodeMetadata:
            def __init__(self, wrappers):
                self.decode_wrappers = wrappers
        class PrefillMetadata:
            def __init__(self, wrappers, use_ragged, extend_no_prefix):
                self.prefill_wrappers = wrappers
        class _Updater:
            def update(self, req_pool_indices, seq_lens, seq_lens_cpu, seq_lens_sum, decode_wrappers=None,
                       encoder_lens=None, spec_info=None, fixed_split_size=None, disable_split_kv=None):
                EVENTS.append(("plan", len(seq_lens), id(decode_wrappers)))
        class FlashInferAttnBackend:
            def __init__(self):
                self.indices_updater_decode = _Updater()
                self.decode_cuda_graph_metadata = {}
                self.forward_metadata = None
                self.disable_cuda_graph_kv_split = False
            def init_forward_metadata_capture_cuda_graph(self, bs, num_tokens, req_pool_indices, seq_lens,
                                                         encoder_lens, forward_mode, spec_info):
                wrappers = [object()]  # SGLang allocates a fresh workspace here
                EVENTS.append(("alloc", bs))
                self.decode_cuda_graph_metadata[bs] = wrappers
                self.forward_metadata = DecodeMetadata(wrappers)
        class FixedWorkspaceBackend:  # fa3-like: metadata are views over one start-up workspace
            def __init__(self):
                self.decode_cuda_graph_metadata = {}
            def init_forward_metadata_capture_cuda_graph(self, bs, *a):
                EVENTS.append(("view", bs))
                self.decode_cuda_graph_metadata[bs] = "view"
    """,
    "sglang/srt/layers/moe/__init__.py": "",
    "sglang/srt/layers/moe/utils.py": """
        import os
        class _Backend:
            def is_deepep(self):
                return os.environ.get("FAKE_DEEPEP") == "1"
        def get_moe_a2a_backend():
            return _Backend()
    """,
    "sglang/srt/layers/moe/token_dispatcher/__init__.py": "",
    "sglang/srt/layers/moe/token_dispatcher/deepep.py": """
        from sglang.srt.layers.attention.flashinfer_backend import EVENTS
        class DeepEPBuffer:
            _buffer = None
        class _LowLatency:
            def _get_buffer(self):
                if DeepEPBuffer._buffer is None:
                    EVENTS.append(("deepep_buffer",))
                    DeepEPBuffer._buffer = object()
                return DeepEPBuffer._buffer
        class DeepEPDispatcher:
            def __init__(self):
                self._low_latency_dispatcher = _LowLatency()
        class MaybeTboDeepEPDispatcher:
            def __init__(self):
                self._inners = [DeepEPDispatcher()]
    """,
}

PREPASS_SCRIPT = r"""
import os, sys, types
sys.path.insert(0, FAKE_ROOT)
sys.path.insert(0, ROOT)
from foundry_b200.integration import runtime
from foundry_b200.integration.sglang import hooks as H, prepass
import sglang.srt.model_executor.model_runner as mr
import sglang.srt.model_executor.cuda_graph_runner as cgr
import sglang.srt.layers.attention.flashinfer_backend as fi
from sglang.srt.layers.moe.token_dispatcher import deepep

SIZES = [1, 2, 4, 8]

class Mode:
    def is_decode_or_idle(self): return True
    def is_target_verify(self): return False
    def is_draft_extend(self): return False

class Adapter:
    def capture(self, is_extend_in_batch):
        fi.EVENTS.append(("adapter_capture", is_extend_in_batch))

class Layer:
    def __init__(self):
        self.dispatcher = deepep.MaybeTboDeepEPDispatcher()

class Model:
    def modules(self):
        return [object(), Layer(), Layer()]

def real_capture(self):
    # the upstream loop: per batch size, metadata init then one forward
    for bs in reversed(self.capture_bs):
        self.attn_backend.init_forward_metadata_capture_cuda_graph(
            bs, bs, self.buffers.req_pool_indices[:bs], self.buffers.seq_lens[:bs], None, Mode(), None)
        fi.EVENTS.append(("forward", bs, H._warmup_pass[0], deepep.DeepEPBuffer._buffer is not None))
    return "captured"
cgr.CudaGraphRunner.capture = real_capture

toml = os.path.join(TMP, MODE + ".toml")
with open(toml, "w") as fh:
    fh.write('mode = "%s"\nbase_addr = "0x620000000000"\nregion_size = "1GB"\nscratch_space_size = "32MB"\n'
             'workspace_root = "%s"\n' % (MODE, os.path.join(TMP, "arch")))
H.install_hooks(toml)
runtime.setup_graph_extension(H._config, 0)

g = cgr.CudaGraphRunner()
g.graphs, g.output_buffers = {"keep": 1}, {}
g.capture_bs = SIZES
g.num_tokens_per_bs = 1
g.capture_forward_mode = Mode()
g.get_spec_info = lambda n: None
g.buffers = types.SimpleNamespace(req_pool_indices=list(range(8)), seq_lens=__import__("torch").ones(8, dtype=__import__("torch").int32),
                                  encoder_lens=None)
g.attn_backend = fi.FlashInferAttnBackend() if BACKEND == "flashinfer" else fi.FixedWorkspaceBackend()
g.model_runner = types.SimpleNamespace(model=Model())
g.deepep_adapter = Adapter()
real_init = g.attn_backend.init_forward_metadata_capture_cuda_graph

# the warm-up flag turns the graph capture into one plain forward
H._warmup_pass[0] = True
assert cgr.CudaGraphRunner._capture_graph(g, None, None, None, lambda: 5) == 5
H._warmup_pass[0] = False

r = g.capture()
ev = fi.EVENTS
allocs = [e[1] for e in ev if e[0] == "alloc"]
deep = os.environ.get("FAKE_DEEPEP") == "1"
if deep:
    assert ev[0] == ("deepep_buffer",), ev  # before any metadata or forward
else:
    assert ("deepep_buffer",) not in ev
if BACKEND == "flashinfer":
    assert allocs == [8, 4, 2, 1], allocs  # pre-pass only, largest first; the loops allocate nothing more
    assert g.attn_backend.init_forward_metadata_capture_cuda_graph == real_init  # shim removed after capture
if MODE == "save":
    assert r == "captured" and g.graphs == {"keep": 1}
    fw = [e for e in ev if e[0] == "forward"]
    if deep:  # a warm-up pass (flag set, buffer already there), then the real loop
        assert [e[1:] for e in fw] == [(b, True, True) for b in (8, 4, 2, 1)] + [(b, False, True) for b in (8, 4, 2, 1)], fw
    else:
        assert [e[1:3] for e in fw] == [(b, False) for b in (8, 4, 2, 1)], fw
    if BACKEND == "flashinfer":
        plans = [e for e in ev if e[0] == "plan"]
        assert len(plans) == len(fw), (plans, fw)  # each loop iteration re-planned a pre-pass wrapper
else:
    assert r is None and not [e for e in ev if e[0] == "forward"]  # LOAD runs no capture loop
    if BACKEND != "flashinfer":
        assert [e[1] for e in ev if e[0] == "view"] == [8, 4, 2, 1]
    assert ("adapter_capture", False) in ev
print("PREPASS_OK", " ".join(repr(e) for e in ev if e[0] in ("alloc", "deepep_buffer")))
H.uninstall_hooks()
"""



@pytest.mark.parametrize("backend", ["flashinfer", "fixed"])
@pytest.mark.parametrize("deep", ["0", "1"])
def test_sglang_prepass_and_deepep_bootstrap(tmp_path, backend, deep):
    """SAVE and LOAD build FlashInfer's per-batch-size metadata in the same
    order before the capture loop / graph load (SAVE's loop then reuses it),
    create the DeepEP buffer first, run SAVE's DeepEP warm-up pass with the
    flag that makes the capture a plain forward, and set DeepEP's captured
    mode after LOAD; fixed-workspace backends get their views after LOAD."""
    fake = tmp_path / "fake"
    _fake_tree(fake)
    for rel, src in PREPASS_FAKE.items():
        p = fake / rel
        p.parent.mkdir(parents=True, exist_ok=True)
        p.write_text(textwrap.dedent(src))
    env = dict(os.environ, FOUNDRY_CUDA_DRIVER=MOCK, PYTHONPATH=ROOT, CUDA_VISIBLE_DEVICES="", FAKE_DEEPEP=deep)
    env.pop("LD_PRELOAD", None)
    outs = {}
    for mode in ("save", "load"):
        code = (f"ROOT={ROOT!r}; TMP={str(tmp_path)!r}; FAKE_ROOT={str(fake)!r}; MODE={mode!r}; "
                f"BACKEND={backend!r}\n" + PREPASS_SCRIPT)
        r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=180)
        assert r.returncode == 0 and "PREPASS_OK" in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]
        outs[mode] = [line for line in r.stdout.splitlines() if line.startswith("PREPASS_OK")][0]
    assert outs["save"] == outs["load"]  # same region-visible steps in the same order
