"""Deterministic VMM allocation region (Python side).

Parity: reference python/foundry/allocation_region.py:31-105. ``parse_size``
accepts the same formats; ``allocation_region`` is the same context manager
(set region -> optional preallocation -> yield -> free -> stop).
"""

from __future__ import annotations

import re
from contextlib import contextmanager

from ._native import core

_SIZE_RE = re.compile(r"^(\d+(?:\.\d+)?)\s*(B|KB|MB|GB|TB|KIB|MIB|GIB|TIB)?$")
_UNITS = {
    "B": 1,
    "KB": 1 << 10, "KIB": 1 << 10,
    "MB": 1 << 20, "MIB": 1 << 20,
    "GB": 1 << 30, "GIB": 1 << 30,
    "TB": 1 << 40, "TIB": 1 << 40,
}


def parse_size(size: int | str) -> int:
    """Parses ``"1.5GB"``, ``"16MB"``, ``"24KB"``, ``"512"`` (binary units) or an int."""
    if isinstance(size, int):
        if size < 0:
            raise ValueError(f"size must be non-negative, got {size}")
        return size
    m = _SIZE_RE.match(size.strip().upper())
    if not m:
        raise ValueError(f"cannot read {size!r} as a size: use a byte count or a number with a binary "
                         "unit (B, KB, MB, GB, TB; KiB..TiB also accepted)")
    return int(float(m.group(1)) * _UNITS[m.group(2) or "B"])


def parse_addr(base: int | str) -> int:
    if isinstance(base, int):
        return base
    s = base.strip().lower()
    return int(s, 16) if s.startswith("0x") else int(s)


def set_allocation_region(base: int | str, size: int | str) -> None:
    core().set_allocation_region(parse_addr(base), parse_size(size))


def stop_allocation_region() -> None:
    core().stop_allocation_region()


def resume_allocation_region() -> None:
    core().resume_allocation_region()


def release_allocation_region() -> None:
    """Unmaps every chunk and frees the reserved span (end of process / tests)."""
    core().release_allocation_region()


def preallocate_region(size: int | str) -> bool:
    return core().preallocate_region(parse_size(size))


def free_preallocated_region() -> None:
    core().free_preallocated_region()


def get_current_alloc_offset() -> int:
    return core().get_current_alloc_offset()


def set_current_alloc_offset(offset: int) -> None:
    core().set_current_alloc_offset(int(offset))


@contextmanager
def allocation_region(base: int | str, size: int | str, prealloc_size: int | str | None = None):
    """Routes allocations into ``[base, base + size)`` for the duration of the block.

    With ``prealloc_size`` the first ``prealloc_size`` bytes are mapped up front
    and later allocations inside that window are pointer bumps.

    Libraries with their own memory pool (torch's caching allocator) keep the
    memory they obtained inside the block after it ends; prefer explicit
    set/stop/resume around the code whose allocations must be deterministic.
    """
    set_allocation_region(base, size)
    try:
        if prealloc_size is not None:
            n = parse_size(prealloc_size)
            if not preallocate_region(n):
                raise RuntimeError(f"Failed to preallocate {n} bytes: {core().last_error()}")
        yield
    finally:
        if prealloc_size is not None:
            free_preallocated_region()
        stop_allocation_region()
