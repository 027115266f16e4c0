"""Tracing: NVTX ranges (visible in Nsight Systems) plus host wall-clock
timings of the named phases of SAVE / LOAD / prefill / capture.

The reference times its restore phases with std::chrono + fprintf and its
Python hooks with ``[foundry TIMING]`` logs (reference
csrc/CUDAGraphParallel.cpp:1853-1858, python/foundry/integration/vllm/hooks.py:106-112);
here every phase is an NVTX range and its duration is kept for reports.
"""

from __future__ import annotations

import os
import sys
import time
from contextlib import contextmanager

_timings: dict[str, list[float]] = {}
_VERBOSE = os.environ.get("FOUNDRY_TRACE", "") not in ("", "0")


def _nvtx():
    try:
        import torch

        if torch.cuda.is_available():
            return torch.cuda.nvtx
    except Exception:  # noqa: BLE001 - tracing must never break the caller
        pass
    return None


@contextmanager
def phase(name: str):
    """NVTX range + wall-clock timing of one named phase."""
    nv = _nvtx()
    if nv is not None:
        nv.range_push(name)
    t0 = time.perf_counter()
    try:
        yield
    finally:
        dt = time.perf_counter() - t0
        if nv is not None:
            nv.range_pop()
        _timings.setdefault(name, []).append(dt)
        if _VERBOSE:
            print(f"[foundry TIMING] {name}: {dt * 1e3:.2f} ms", file=sys.stderr)


def timings(reset: bool = False) -> dict[str, dict]:
    """{phase: {"n", "total_s", "last_s"}} of the phases seen so far."""
    out = {k: {"n": len(v), "total_s": sum(v), "last_s": v[-1]} for k, v in _timings.items()}
    if reset:
        _timings.clear()
    return out


__all__ = ["phase", "timings"]
