"""Creates the CUDA primary context on a background thread while the process
is still importing torch.

A fresh LOAD process spends most of its time to the first token importing
Python modules (torch above all) and creating the device's CUDA context;
neither needs the other. When ``FOUNDRY_EARLY_CUDA_INIT=<device ordinal>`` is
set, importing ``foundry_b200`` starts a thread that calls ``cuInit``,
``cuDeviceGet`` and ``cuDevicePrimaryCtxRetain`` through ctypes (ctypes
releases the GIL for the duration of each call), so the context is built
while the main thread imports torch. torch later binds the same primary
context (the runtime API uses it), finding it already created. The retain is
never released: the context lives as long as the process, as torch's does.

The runner's ``load`` and ``serve`` commands are started with the variable
set by ``bench.py``; nothing else sets it.

Parity: no counterpart in the reference, whose cold start is vLLM's or
SGLang's own process start.
"""

from __future__ import annotations

import ctypes
import os
import threading
import time

ENV = "FOUNDRY_EARLY_CUDA_INIT"
_thread: threading.Thread | None = None
_result: dict = {}


def _run(ordinal: int) -> None:
    t0 = time.perf_counter()
    try:
        lib = ctypes.CDLL("libcuda.so.1")
        rc = lib.cuInit(0)
        dev = ctypes.c_int(0)
        if rc == 0:
            rc = lib.cuDeviceGet(ctypes.byref(dev), ordinal)
        ctx = ctypes.c_void_p()
        if rc == 0:
            rc = lib.cuDevicePrimaryCtxRetain(ctypes.byref(ctx), dev)
        _result.update(device=ordinal, rc=int(rc), seconds=round(time.perf_counter() - t0, 4))
    except OSError as e:  # no driver library (a CPU box)
        _result.update(device=ordinal, error=str(e))


def start_from_env() -> bool:
    """Starts the thread if ``FOUNDRY_EARLY_CUDA_INIT`` names a device."""
    global _thread
    v = os.environ.get(ENV)
    if _thread is not None or not v:
        return False
    try:
        ordinal = int(v)
    except ValueError:
        return False
    _thread = threading.Thread(target=_run, args=(ordinal,), name="foundry-early-cuda", daemon=True)
    _thread.start()
    return True


def result(timeout: float = 30.0) -> dict | None:
    """Waits for the thread; its outcome (None when it was never started)."""
    if _thread is None:
        return None
    _thread.join(timeout)
    return dict(_result)
