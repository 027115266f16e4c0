"""SGLang integration: persist the CUDA graphs of SGLang's CudaGraphRunner.

``install_hooks(config)`` patches ``CudaGraphRunner.capture_one_batch_size``
(graph capture of one decode batch size) to capture + save (SAVE) or restore
(LOAD) through foundry_b200.integration.graph_ops, keyed by the batch size,
and ``CudaGraphRunner.capture`` to start all builds first (LOAD) or write the
manifest, packed modules and final offset after (SAVE). Region setup runs from
``ModelRunner.init_torch_distributed`` (after the communicator init).

Parity: reference python/foundry/integration/sglang/hooks.py:67-594. SGLang
is not installed on this build's image, so these patches are not exercised
here; ``install_hooks`` raises a clear error when the patch targets are absent.
"""

from __future__ import annotations

import os

from .. import graph_ops, runtime
from ..config import GraphExtensionConfig, GraphExtensionMode

_originals: dict = {}
_config: GraphExtensionConfig | None = None


def _targets():
    try:
        from sglang.srt.model_executor import cuda_graph_runner as cgr
        from sglang.srt.model_executor import model_runner as mr
    except ImportError as e:  # pragma: no cover - depends on the image
        raise ImportError("SGLang is not installed: the SGLang graph extension cannot be installed") from e
    for cls, name in ((cgr.CudaGraphRunner, "capture_one_batch_size"), (cgr.CudaGraphRunner, "capture"),
                      (mr.ModelRunner, "init_torch_distributed")):
        if not hasattr(cls, name):
            raise ImportError(f"this SGLang has no {cls.__name__}.{name}: unsupported version")
    return cgr, mr


def _capture_one_batch_size(self, bs, forward, *a, **k):
    if runtime.mode() == GraphExtensionMode.NONE:
        return _originals["capture_one_batch_size"](self, bs, forward, *a, **k)
    key = graph_ops.GraphKey("FULL", int(bs), int(bs), True, False, None)
    # SGLang's forward closure reads its static buffers; capture it as is.
    return graph_ops.capture_or_load(key, forward, pool=getattr(self, "graph_memory_pool", None),
                                     stream=getattr(self, "stream", None))


def _capture(self, *a, **k):
    st = runtime.state()
    if st is not None and st.config.mode == GraphExtensionMode.LOAD:
        graph_ops.start_graph_builds(st.config.workspace_dir)
    r = _originals["capture"](self, *a, **k)
    if st is not None and st.config.mode == GraphExtensionMode.SAVE:
        graph_ops.finalize_save()
    if st is not None and st.config.mode != GraphExtensionMode.NONE:
        runtime.capture_final_alloc_offset()
    return r


def _init_torch_distributed(self, *a, **k):
    r = _originals["init_torch_distributed"](self, *a, **k)
    dp = int(getattr(self, "dp_rank", 0) or 0)
    tp_size = int(getattr(self, "tp_size", 1) or 1)
    runtime.setup_graph_extension(_config, dp * tp_size + int(getattr(self, "tp_rank", 0) or 0))
    if _config.mode != GraphExtensionMode.NONE:
        runtime.skip_to_scratch_boundary()
    return r


def install_hooks(config: GraphExtensionConfig | str) -> None:
    global _config
    if isinstance(config, (str, os.PathLike)):
        config = GraphExtensionConfig.from_toml(config)
    _config = config
    if _originals:
        return
    cgr, mr = _targets()
    _originals["capture_one_batch_size"] = cgr.CudaGraphRunner.capture_one_batch_size
    _originals["capture"] = cgr.CudaGraphRunner.capture
    _originals["init_torch_distributed"] = mr.ModelRunner.init_torch_distributed
    cgr.CudaGraphRunner.capture_one_batch_size = _capture_one_batch_size
    cgr.CudaGraphRunner.capture = _capture
    mr.ModelRunner.init_torch_distributed = _init_torch_distributed


def uninstall_hooks() -> None:
    if not _originals:
        return
    cgr, mr = _targets()
    cgr.CudaGraphRunner.capture_one_batch_size = _originals.pop("capture_one_batch_size")
    cgr.CudaGraphRunner.capture = _originals.pop("capture")
    mr.ModelRunner.init_torch_distributed = _originals.pop("init_torch_distributed")
    runtime.reset()


__all__ = ["install_hooks", "uninstall_hooks"]
