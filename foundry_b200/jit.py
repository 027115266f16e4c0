"""Persisting kernels that a JIT compiler (Triton, and so torch.compile /
Inductor) builds in this process.

A Triton kernel is compiled from Python source on this machine and handed to
the driver as a cubin held in memory (``cuModuleLoadData``). The interposer
alone cannot tell how long such a heap image is without reading its headers,
which this project never does; the loaders above it, however, hold the exact
bytes they load. After a kernel is loaded, this module passes its module
handle and those bytes to the registry (``fb_registry_adopt_module``): the
image is hashed and kept like one of this repository's own cubins, captured
graphs name its kernels by (hash, entry name), the archive's pack holds the
bytes, and a LOAD process reloads them with ``cuLibraryLoadData`` without
compiling anything (it need not import Triton or Inductor at all).

Two loaders are wrapped, each as soon as its module is imported (or when
``foundry_b200`` is imported, if it already is), so kernels loaded before the
first capture (a torch.compile warm-up) are adopted too:

* ``triton.compiler.compiler.CompiledKernel._init_handles``: Triton's own
  launcher; the object keeps the module handle and the cubin bytes.
* ``torch._inductor.runtime.static_triton_launcher.StaticallyLaunchedTritonKernel.load_kernel``:
  Inductor's static launcher, which loads the cubin that Triton compiled for
  it (``cubin_raw`` in memory, else the file Triton wrote) and keeps only the
  function handle; the module comes from ``cuFuncGetModule``.

``adopt_loaded_kernel`` can also be called directly with any object that has
``module`` and ``kernel`` (bytes).

Parity: reference csrc/hook.cpp:558-727 (captures every image passed to
cuModuleLoadData* by reading its container headers); its core test persists
a torch.compile'd model (tests/test_load_graph.py:36-89).
"""

from __future__ import annotations

import importlib.abc
import importlib.util
import sys
import threading

from ._native import core

_lock = threading.Lock()
adopted: dict[int, int] = {}  # module or function handle -> image hash
_patched: set[str] = set()


def adopt_loaded_kernel(kernel) -> int | None:
    """Registers a loaded Triton kernel's image (``kernel.module`` handle and
    ``kernel.kernel`` cubin bytes); returns the image hash, or None when the
    object has no loaded module or no binary bytes."""
    mod = getattr(kernel, "module", None)
    image = getattr(kernel, "kernel", None)
    if not mod or not isinstance(image, (bytes, bytearray)) or not image:
        return None
    mod = int(mod)
    h = adopted.get(mod)
    if h is None:
        h = core().adopt_jit_module(mod, bytes(image))
        adopted[mod] = h
    return h


def adopt_loaded_function(function: int, image: bytes) -> int:
    """Registers the image that ``function`` (a CUfunction handle) was loaded from."""
    h = adopted.get(function)
    if h is None:
        h = core().adopt_jit_function(int(function), bytes(image))
        adopted[function] = h
    return h


def _patch_triton(module) -> None:
    cls = getattr(module, "CompiledKernel", None)
    if cls is None or getattr(cls._init_handles, "_foundry_adopts", False):
        return
    original = cls._init_handles

    def _init_handles(self):
        loaded_before = self.module is not None
        original(self)
        if not loaded_before and self.module is not None:
            adopt_loaded_kernel(self)

    _init_handles._foundry_adopts = True
    cls._init_handles = _init_handles


def _patch_inductor(module) -> None:
    cls = getattr(module, "StaticallyLaunchedTritonKernel", None)
    if cls is None or getattr(cls.load_kernel, "_foundry_adopts", False):
        return
    original = cls.load_kernel

    def load_kernel(self, device: int) -> None:
        if getattr(self, "function", None) is not None:
            return original(self, device)
        image = getattr(self, "cubin_raw", None)
        if image is None and getattr(self, "cubin_path", None):
            with open(self.cubin_path, "rb") as f:  # the cubin Triton compiled for this kernel
                image = f.read()
        original(self, device)
        if image and self.function:
            adopt_loaded_function(int(self.function), image)

    load_kernel._foundry_adopts = True
    cls.load_kernel = load_kernel


_TARGETS = {
    "triton.compiler.compiler": _patch_triton,
    "torch._inductor.runtime.static_triton_launcher": _patch_inductor,
}


def _apply(name: str, module) -> None:
    with _lock:
        _TARGETS[name](module)
        _patched.add(name)


class _AfterImport(importlib.abc.MetaPathFinder):
    """Patches each target module right after it is first imported."""

    def find_spec(self, name, path, target=None):
        if name not in _TARGETS or name in _patched:
            return None
        sys.meta_path.remove(self)  # keeps find_spec below from recursing into this finder
        try:
            spec = importlib.util.find_spec(name)
        finally:
            sys.meta_path.insert(0, self)
        if spec is None or spec.loader is None:
            return None
        inner = spec.loader

        class _Loader(importlib.abc.Loader):
            def create_module(self, spec):
                return inner.create_module(spec)

            def exec_module(self, module):
                inner.exec_module(module)
                _apply(name, module)

        spec.loader = _Loader()
        return spec


def install() -> None:
    """Adopts every JIT kernel loaded from now on (idempotent)."""
    for name in _TARGETS:
        mod = sys.modules.get(name)
        if mod is not None:
            _apply(name, mod)
    if len(_patched) < len(_TARGETS) and not any(isinstance(f, _AfterImport) for f in sys.meta_path):
        sys.meta_path.insert(0, _AfterImport())


def installed() -> bool:
    """True once at least one JIT loader is wrapped."""
    return bool(_patched)
