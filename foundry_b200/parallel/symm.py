"""Symmetric device memory across the ranks of one node.

Every rank allocates ``size`` bytes with cuMemCreate (POSIX-fd shareable),
the fds are exchanged over Unix-domain sockets (SCM_RIGHTS - an fd number is
only meaningful inside its own process), and every process maps rank r's
allocation at ``base + r * stride``. Peer pointers are therefore identical
numbers in every process, and - because ``base`` is fixed - identical across
SAVE and LOAD, so CUDA graphs that captured peer pointers stay valid after a
restore. Where NVSwitch multicast (NVLS) is available, a multicast object
over all ranks' buffers is mapped at ``base + world * stride``: one
``multimem`` store there reaches every GPU, one ``multimem.ld_reduce`` returns
the sum over GPUs.

Parity: the reference maps IPC'd VMM memory at the exporter's address
(csrc/hook.cpp:2864-3080) and relies on NVSHMEM (DeepEP) for symmetric heaps;
this is our own substrate.
"""

from __future__ import annotations

import os
import socket
import struct
import tempfile
import threading
import time

import torch
import torch.distributed as dist

from .._native import core

DEFAULT_BASE = 0x700000000000
CTRL_BYTES = 4096  # barrier flags + epoch counter at the start of each rank's buffer

_instances = 0


def _recv_exact(conn, n):
    buf = b""
    while len(buf) < n:
        chunk = conn.recv(n - len(buf))
        if not chunk:
            raise ConnectionError("peer closed the fd-exchange socket")
        buf += chunk
    return buf


def exchange_fds(my_fd: int, rank: int, world: int, tag: str, group=None, timeout: float = 60.0) -> dict[int, int]:
    """Sends ``my_fd`` to every other rank and returns {rank: fd} (fds valid in this process)."""
    path = os.path.join(tempfile.gettempdir(), f"fb_symm_{tag}_{rank}.sock")
    if os.path.exists(path):
        os.unlink(path)
    srv = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
    srv.bind(path)
    srv.listen(world)
    srv.settimeout(timeout)
    got: dict[int, int] = {}
    err: list[BaseException] = []

    def serve():
        try:
            for _ in range(world - 1):
                conn, _ = srv.accept()
                with conn:
                    conn.settimeout(timeout)
                    msg, fds, _, _ = socket.recv_fds(conn, 4, 1)
                    if len(msg) < 4:
                        msg += _recv_exact(conn, 4 - len(msg))
                    if not fds:
                        raise ConnectionError("no fd received")
                    got[struct.unpack("<i", msg[:4])[0]] = fds[0]
        except BaseException as e:  # surfaced below
            err.append(e)

    th = threading.Thread(target=serve, daemon=True)
    th.start()
    dist.barrier(group=group)
    for peer in range(world):
        if peer == rank:
            continue
        peer_path = os.path.join(tempfile.gettempdir(), f"fb_symm_{tag}_{peer}.sock")
        deadline = time.time() + timeout
        while True:
            try:
                c = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
                c.settimeout(timeout)
                c.connect(peer_path)
                break
            except (FileNotFoundError, ConnectionRefusedError):
                c.close()
                if time.time() > deadline:
                    raise TimeoutError(f"rank {peer} did not open its fd-exchange socket")
                time.sleep(0.01)
        with c:
            socket.send_fds(c, [struct.pack("<i", rank)], [my_fd])
    th.join(timeout)
    srv.close()
    os.unlink(path)
    if err:
        raise err[0]
    if len(got) != world - 1:
        raise TimeoutError(f"received {len(got)} of {world - 1} peer fds")
    dist.barrier(group=group)
    return got


class SymmetricMemory:
    """``size`` bytes per rank, mapped at base + r * stride in every process."""

    def __init__(self, size: int, group=None, base: int = DEFAULT_BASE, multicast: bool = True,
                 device: int | None = None):
        global _instances
        c = core()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.mock = c.driver_is_mock()  # CPU tests: host memory stands in for device memory
        if device is None:
            device = 0 if self.mock else torch.cuda.current_device()
        self.device = device
        gran = c.vmm_granularity(self.device)
        self.multicast = bool(multicast) and c.mc_supported() and self.world > 1
        if self.multicast:
            try:
                gran = max(gran, c.mc_granularity(self.world, size))
            except RuntimeError:
                self.multicast = False
        self.size = -(-max(size, CTRL_BYTES) // gran) * gran
        self.stride = self.size
        self.base = base
        span = self.stride * (self.world + (1 if self.multicast else 0))
        tag_box = [f"{os.getpid()}_{_instances}"]
        _instances += 1
        dist.broadcast_object_list(tag_box, src=0, group=group)
        tag = tag_box[0]

        self.handle = c.vmm_create(self.size, self.device)
        self.va = c.vmm_reserve(base, span, gran)
        self.span = span
        my_fd = c.vmm_export_fd(self.handle)
        fds = exchange_fds(my_fd, self.rank, self.world, tag + "_mem", group)
        os.close(my_fd)
        self.peer_handles = {self.rank: self.handle}
        for r, fd in fds.items():
            self.peer_handles[r] = c.vmm_import_fd(fd)
            os.close(fd)
        for r in range(self.world):
            c.vmm_map(self.ptr(r), self.size, self.peer_handles[r], 0)
            c.vmm_set_access(self.ptr(r), self.size, [self.device])
        self.mc_handle = 0
        if self.multicast:
            self._setup_multicast(tag)
        # zero the control block (flags, epoch)
        if self.mock:
            import ctypes

            ctypes.memset(self.local_ptr, 0, CTRL_BYTES)
        else:
            self.tensor(self.rank, (CTRL_BYTES,), torch.uint8).zero_()
            torch.cuda.synchronize()
        dist.barrier(group=group)

    def _setup_multicast(self, tag: str) -> None:
        c = core()
        if self.rank == 0:
            self.mc_handle = c.mc_create(self.world, self.size)
            fd = c.vmm_export_fd(self.mc_handle)
        else:
            fd = -1
        # only rank 0's fd matters: everybody exchanges, rank 0 sends the real one
        dummy = os.open("/dev/null", os.O_RDONLY) if fd < 0 else fd
        fds = exchange_fds(dummy, self.rank, self.world, tag + "_mc", self.group)
        os.close(dummy)
        if self.rank != 0:
            self.mc_handle = c.vmm_import_fd(fds[0])
        for f in fds.values():
            os.close(f)
        c.mc_add_device(self.mc_handle, self.device)
        dist.barrier(group=self.group)
        c.mc_bind_mem(self.mc_handle, 0, self.handle, 0, self.size)
        dist.barrier(group=self.group)
        c.vmm_map(self.mc_ptr, self.size, self.mc_handle, 0)
        c.vmm_set_access(self.mc_ptr, self.size, [self.device])

    # ---- addressing ------------------------------------------------------------------------
    def ptr(self, r: int, offset: int = 0) -> int:
        return self.base + r * self.stride + offset

    @property
    def local_ptr(self) -> int:
        return self.ptr(self.rank)

    @property
    def mc_ptr(self) -> int:
        return self.base + self.world * self.stride if self.multicast else 0

    def tensor(self, r: int, shape, dtype, offset: int = 0) -> torch.Tensor:
        from ..graphs import tensor_from_ptr

        shape = tuple(shape)
        strides, acc = [], 1
        for s in reversed(shape):
            strides.append(acc)
            acc *= s
        return tensor_from_ptr(self.ptr(r, offset), shape, tuple(reversed(strides)), dtype)

    def layout(self) -> dict:
        return {"base": self.base, "stride": self.stride, "world": self.world, "multicast": self.multicast}

    def close(self) -> None:
        c = core()
        if not self.mock:
            torch.cuda.synchronize()
        for r in range(self.world):
            c.vmm_unmap(self.ptr(r), self.size)
        if self.multicast:
            c.vmm_unmap(self.mc_ptr, self.size)
            c.mc_unbind(self.mc_handle, self.device, 0, self.size)
            c.vmm_release(self.mc_handle)
        for r, h in self.peer_handles.items():
            c.vmm_release(h)
        c.vmm_free_va(self.va, self.span)
