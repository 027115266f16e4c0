"""Static device arena carved from the deterministic VMM region.

Every persistent buffer of the runner (weights, KV cache, activations,
workspaces) is a view into chunks allocated with the region's cursor
allocator, in a fixed order, so the same model/config produces the same
device addresses in the SAVE process and in every LOAD process. That is what
makes the pointers baked into captured graphs valid after a restore, without
replaying any allocator history.

Without a region (``base=None``) the arena falls back to ordinary torch
allocations: everything works except persistence.
"""

from __future__ import annotations

import math

import torch

from .._native import core
from ..allocation_region import parse_size
from ..graphs import tensor_from_ptr

_ALIGN = 256


class Arena:
    def __init__(self, base: int | None, size: int | str, device=None, chunk: int | str = "1GB"):
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.base = base
        self.size = parse_size(size)
        self.chunk = parse_size(chunk)
        self._chunks: list[tuple[int, int]] = []  # (ptr, size)
        self._cur_ptr = 0
        self._cur_left = 0
        self._owned: list[torch.Tensor] = []  # fallback allocations
        self.used = 0
        if base is not None:
            if self.device.type == "cuda":  # (a CPU device: host-side layout checks on the mock driver)
                torch.cuda.init()
            c = core()
            c.set_allocation_region(base, self.size)

    @property
    def persistent(self) -> bool:
        return self.base is not None

    def _new_chunk(self, nbytes: int) -> None:
        n = max(self.chunk, nbytes)
        gran = core().region_granularity()
        n = math.ceil(n / gran) * gran
        ptr = core().region_alloc(n)
        self._chunks.append((ptr, n))
        self._cur_ptr, self._cur_left = ptr, n

    def alloc_bytes(self, nbytes: int) -> int:
        nbytes = math.ceil(max(nbytes, 1) / _ALIGN) * _ALIGN
        if nbytes > self._cur_left and nbytes >= self.chunk // 4:
            # Large tensors (KV-cache layers, weight matrices) get a region
            # allocation of their own, rounded to the granularity only: carving
            # them out of fixed-size chunks strands the chunk tails (a 605 MB
            # KV layer per 1 GB chunk wastes 40% of the device).
            gran = core().region_granularity()
            n = math.ceil(nbytes / gran) * gran
            ptr = core().region_alloc(n)
            self._chunks.append((ptr, n))
            self.used += nbytes
            return ptr
        if nbytes > self._cur_left:
            self._new_chunk(nbytes)
        p = self._cur_ptr
        self._cur_ptr += nbytes
        self._cur_left -= nbytes
        self.used += nbytes
        return p

    def empty(self, shape, dtype=torch.bfloat16) -> torch.Tensor:
        shape = tuple(int(s) for s in shape)
        numel = math.prod(shape)
        esize = torch.empty((), dtype=dtype).element_size()
        if not self.persistent:
            t = torch.empty(shape, dtype=dtype, device=self.device)
            self.used += numel * esize
            return t
        ptr = self.alloc_bytes(numel * esize)
        strides = []
        acc = 1
        for s in reversed(shape):
            strides.append(acc)
            acc *= s
        return tensor_from_ptr(ptr, shape, tuple(reversed(strides)), dtype)

    def zeros(self, shape, dtype=torch.bfloat16) -> torch.Tensor:
        t = self.empty(shape, dtype)
        t.zero_()
        return t

    def release(self) -> None:
        """Unmaps everything (only at the end of a process or test)."""
        if self.persistent:
            torch.cuda.synchronize()
            core().release_allocation_region()
            self._chunks.clear()
