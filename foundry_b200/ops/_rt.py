"""Kernel runtime: loads this repository's sm_100a cubins through the module
registry and launches their entry points with ``cuLaunchKernelEx``.

Every op in ``foundry_b200.ops`` goes through here. Loading through the
registry gives each image a content hash, which is what lets a captured
graph name its kernels as (hash, entry) and find them again in a fresh
process. A missing cubin or a CPU-only process raises immediately: there is
no fallback path.
"""

from __future__ import annotations

import contextlib
import os
import threading

import torch

from .._native import KERNEL_DIR, core

IMAGES = ("gemm_bf16", "elementwise", "attention", "gemm_fp8", "moe", "comm")

_lock = threading.Lock()
_images: dict[str, int] = {}
_funcs: dict[tuple[str, str, int], int] = {}


def image_hash(image: str) -> int:
    h = _images.get(image)
    if h is not None:
        return h
    with _lock:
        h = _images.get(image)
        if h is None:
            path = KERNEL_DIR / f"{image}.cubin"
            if not path.exists():
                raise RuntimeError(
                    f"kernel image {path} is missing; build with `python -m foundry_b200._build`"
                )
            if not torch.cuda.is_available() and not core().driver_is_mock():
                raise RuntimeError("foundry_b200 kernels need a CUDA device")
            if torch.cuda.is_available():
                torch.cuda.init()  # make the primary context current on this thread
            _, h = core().load_image_file(str(path))
            _images[image] = h
    return h


def function(image: str, name: str, smem: int = 0) -> int:
    key = (image, name, smem)
    f = _funcs.get(key)
    if f is None:
        f = core().get_function(image_hash(image), name, smem if smem > 48 * 1024 else 0)
        _funcs[key] = f
    return f


# Programmatic dependent launch: inside ``pdl()`` the kernels of these images
# are launched with programmatic stream serialization, so each may start (and
# run its set-up) while the previous kernel of the stream finishes; every
# kernel of these images calls griddepcontrol.wait before it touches memory
# another kernel writes (csrc/kernels/fb_common.cuh). Kernels of other images
# (the peer-memory collectives, MoE) launch in plain stream order. Set
# FOUNDRY_PDL=0 to launch everything in plain order.
PDL_IMAGES = frozenset({"elementwise", "attention", "attention_tc", "gemm_bf16"})
PDL_ENABLED = os.environ.get("FOUNDRY_PDL", "1") != "0"
_pdl = threading.local()


@contextlib.contextmanager
def pdl():
    """Launches in this block (this thread) may use programmatic dependent
    launch. Used around the decode step, whose weights no kernel writes."""
    depth = getattr(_pdl, "depth", 0)
    _pdl.depth = depth + 1
    try:
        yield
    finally:
        _pdl.depth = depth


def pdl_active() -> bool:
    return PDL_ENABLED and getattr(_pdl, "depth", 0) > 0


def launch(image: str, name: str, grid, block, args, smem: int = 0, stream: int | None = None,
           cluster=()) -> None:
    if stream is None:
        stream = torch.cuda.current_stream().cuda_stream
    fn = function(image, name, smem)
    core().launch(fn, tuple(grid), tuple(block), smem, stream, args, tuple(cluster),
                  pdl_active() and image in PDL_IMAGES)


def status(image: str) -> int:
    """The image's device status word (0 = healthy; bits = bounded-wait timeouts)."""
    ptr, _ = core().get_global(image_hash(image), "fb_status")
    from ..graphs import tensor_from_ptr

    return int(tensor_from_ptr(ptr, (1,), (1,), torch.int32).item())


def clear_status(image: str) -> None:
    ptr, _ = core().get_global(image_hash(image), "fb_status")
    from ..graphs import tensor_from_ptr

    tensor_from_ptr(ptr, (1,), (1,), torch.int32).zero_()


def loaded_images() -> dict[str, int]:
    return dict(_images)


def sm_count() -> int:
    return torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
