"""SGLang state that captured graphs point into but that SGLang creates
lazily: the per-batch-size attention metadata of FlashInfer and the DeepEP
communication buffer.

Both must exist at the same addresses in SAVE and in LOAD, and both would
otherwise be created at points that differ between the two runs (LOAD runs
no capture loop; SAVE runs no warm-up forwards), so the hooks create them
at fixed points instead:

* Attention metadata. SGLang's FlashInfer backend builds, for every captured
  batch size, decode wrappers that own an integer workspace tensor; the
  captured attention kernels read their plan from it. SGLang allocates them
  inside its capture loop (``init_forward_metadata_capture_cuda_graph``), one
  batch size at a time, interleaved with the graph-pool allocations of each
  capture. ``attention_metadata_prepass`` builds all of them up front, in the
  order of the capture loop (largest batch first), in both SAVE and LOAD, so
  they take the same region offsets. During SAVE's capture loop
  ``ReusePrepassMetadata`` stands in for the backend's init: for a batch size
  whose wrappers already exist it re-plans them in place (no allocation) and
  makes them the forward's metadata. Backends whose graph metadata lives in
  one workspace allocated once at start-up (fa3 and the like) need no
  pre-pass; LOAD only fills their per-batch-size views after the graphs are
  restored, since LOAD replaces the loop that would have filled them.
* DeepEP. The DeepEP buffer (NVSHMEM runtime plus symmetric heap) is created
  on the first MoE dispatch. SAVE suppresses the warm-up forwards where that
  normally happens, and creating it inside a stream capture fails, so
  ``ensure_deepep_buffer`` creates it before the capture (SAVE) or the graph
  load (LOAD), at the same point of both runs. It is a collective over the EP
  group; every rank reaches the capture hook, so every rank calls it.

SGLang's class and attribute names used here (``attn_backend``,
``indices_updater_decode``, ``decode_cuda_graph_metadata``,
``DeepEPDispatcher`` and its ``_get_buffer``, ...) are SGLang's own API.

Parity: reference python/foundry/integration/sglang/graph_ops.py:181-284
and hooks.py:344-547 (the same two problems; the pre-pass order, largest
batch first, is the one SGLang's capture loop uses, so it has to match).
"""

from __future__ import annotations

import importlib
import logging
import time

log = logging.getLogger("foundry")

_FLASHINFER = "sglang.srt.layers.attention.flashinfer_backend"


def uses_per_batch_metadata(attn_backend) -> bool:
    """True for backends that allocate attention metadata per captured batch
    size (FlashInfer: its decode index updater is the marker)."""
    return hasattr(attn_backend, "indices_updater_decode")


def _capture_args(runner, bs: int) -> tuple:
    """Arguments of ``init_forward_metadata_capture_cuda_graph`` for batch
    size ``bs``: the same buffer slices SGLang's capture loop passes."""
    buf = runner.buffers
    num_tokens = bs * runner.num_tokens_per_bs
    encoder_lens = buf.encoder_lens[:bs] if getattr(runner, "is_encoder_decoder", False) else None
    return (bs, num_tokens, buf.req_pool_indices[:bs], buf.seq_lens[:bs], encoder_lens,
            runner.capture_forward_mode, runner.get_spec_info(num_tokens))


def attention_metadata_prepass(runner, init=None) -> int:
    """Builds the attention metadata of every captured batch size, largest
    first; returns how many. ``init`` defaults to the backend's own
    ``init_forward_metadata_capture_cuda_graph``."""
    init = init or runner.attn_backend.init_forward_metadata_capture_cuda_graph
    sizes = sorted(runner.capture_bs, reverse=True)
    for bs in sizes:
        init(*_capture_args(runner, bs))
    return len(sizes)


class ReusePrepassMetadata:
    """SAVE-time stand-in for the FlashInfer backend's
    ``init_forward_metadata_capture_cuda_graph`` that reuses the pre-pass's
    wrappers. Decode (and idle) batches re-plan the decode wrappers of their
    batch size; target-verify and draft-extend batches the prefill wrappers;
    anything else, or a batch size the pre-pass did not build, goes to the
    backend's own init."""

    def __init__(self, backend, real_init):
        self.backend = backend
        self.real_init = real_init
        self.reused = 0

    def __call__(self, bs, num_tokens, req_pool_indices, seq_lens, encoder_lens, forward_mode, spec_info):
        be = self.backend
        if forward_mode.is_decode_or_idle():
            wrappers = be.decode_cuda_graph_metadata.get(bs)
            if wrappers is not None:
                be.indices_updater_decode.update(
                    req_pool_indices, seq_lens, seq_lens.cpu(), int(seq_lens.sum().item()),
                    decode_wrappers=wrappers, encoder_lens=encoder_lens, spec_info=spec_info,
                    fixed_split_size=None, disable_split_kv=getattr(be, "disable_cuda_graph_kv_split", False))
                be.forward_metadata = importlib.import_module(_FLASHINFER).DecodeMetadata(wrappers)
                self.reused += 1
                return None
        elif forward_mode.is_target_verify() or forward_mode.is_draft_extend():
            wrappers = getattr(be, "prefill_cuda_graph_metadata", {}).get(bs)
            if wrappers is not None:
                be.indices_updater_prefill.update(
                    req_pool_indices, seq_lens, seq_lens.cpu(), int(seq_lens.sum().item()), prefix_lens=None,
                    prefill_wrappers=wrappers, use_ragged=False, encoder_lens=encoder_lens, spec_info=spec_info)
                be.forward_metadata = importlib.import_module(_FLASHINFER).PrefillMetadata(wrappers, False, False)
                self.reused += 1
                return None
        return self.real_init(bs, num_tokens, req_pool_indices, seq_lens, encoder_lens, forward_mode, spec_info)


def install_reuse(runner) -> "callable":
    """SAVE: runs the pre-pass and points the backend's capture init at
    ``ReusePrepassMetadata``; returns the function that puts it back."""
    be = runner.attn_backend
    real = be.init_forward_metadata_capture_cuda_graph
    n = attention_metadata_prepass(runner, real)
    be.forward_metadata = None  # the pre-pass's last batch size is no capture's metadata
    shim = ReusePrepassMetadata(be, real)
    be.init_forward_metadata_capture_cuda_graph = shim
    log.info("[foundry] SGLang attention metadata built for %d batch sizes before capture", n)

    def restore():
        be.init_forward_metadata_capture_cuda_graph = real
        log.info("[foundry] SGLang capture reused pre-pass attention metadata %d times", shim.reused)

    return restore


def deepep_active() -> bool:
    """True when SGLang's MoE all-to-all backend is DeepEP."""
    try:
        utils = importlib.import_module("sglang.srt.layers.moe.utils")
        return bool(utils.get_moe_a2a_backend().is_deepep())
    except (ImportError, AttributeError):
        return False


def _deepep_impls(model, dispatcher_cls):
    """DeepEP dispatcher implementations found on the model's modules: a
    module's ``dispatcher`` is a DeepEPDispatcher or a wrapper that holds
    them in ``_inners``; each has a low-latency and/or a normal impl."""
    for module in model.modules():
        d = getattr(module, "dispatcher", None)
        if d is None:
            continue
        for cand in (d, *getattr(d, "_inners", ())):
            if not isinstance(cand, dispatcher_cls):
                continue
            for attr in ("_low_latency_dispatcher", "_normal_dispatcher"):
                impl = getattr(cand, attr, None)
                if impl is not None:
                    yield impl


def ensure_deepep_buffer(runner) -> bool:
    """Creates SGLang's process-wide DeepEP buffer now, outside any stream
    capture, if DeepEP is the all-to-all backend and the buffer does not
    exist yet. Returns True when the buffer exists afterwards."""
    if not deepep_active():
        return False
    mod = importlib.import_module("sglang.srt.layers.moe.token_dispatcher.deepep")
    if getattr(mod.DeepEPBuffer, "_buffer", None) is not None:
        return True
    t0 = time.perf_counter()
    for impl in _deepep_impls(runner.model_runner.model, mod.DeepEPDispatcher):
        impl._get_buffer()  # one impl creates the singleton every impl shares
        log.info("[foundry] DeepEP buffer created before capture in %.3f s", time.perf_counter() - t0)
        return True
    log.warning("[foundry] DeepEP is the all-to-all backend but no DeepEP dispatcher was found on the model; "
                "the buffer will be created lazily (inside the capture, where it fails)")
    return False


__all__ = ["ReusePrepassMetadata", "attention_metadata_prepass", "deepep_active", "ensure_deepep_buffer",
           "install_reuse", "uses_per_batch_metadata"]
