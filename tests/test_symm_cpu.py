"""Symmetric-memory host logic on CPU: two gloo ranks on the mock driver
exchange POSIX fds (SCM_RIGHTS), map each other's allocations at identical
addresses and see each other's writes."""

import ctypes
import os
import socket
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
MOCK = os.path.join(ROOT, "foundry_b200", "lib", "libfoundry_mockcuda.so")

WORKER = r"""
import ctypes, os, sys
import torch.distributed as dist
sys.path.insert(0, ROOT)
dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % PORT, rank=RANK, world_size=2)
from foundry_b200.parallel.symm import SymmetricMemory, CTRL_BYTES
c = __import__("foundry_b200").core()
c.set_allocation_region(0x600000000000, 1 << 30)  # makes a current context on the mock
s = SymmetricMemory(8 << 20, multicast=False)
assert s.ptr(0) == 0x700000000000 and s.ptr(1) == 0x700000000000 + s.stride
msg = ("hello from rank %d" % RANK).encode()
ctypes.memmove(s.local_ptr + CTRL_BYTES, msg, len(msg))
dist.barrier()
peer = 1 - RANK
got = ctypes.string_at(s.ptr(peer) + CTRL_BYTES, len(msg))
assert got == ("hello from rank %d" % peer).encode(), got
# writes into a peer's mapping land in the peer's memory
ctypes.memmove(s.ptr(peer) + CTRL_BYTES + 4096, b"X" * 8, 8)
dist.barrier()
assert ctypes.string_at(s.local_ptr + CTRL_BYTES + 4096, 8) == b"X" * 8
s.close()
dist.destroy_process_group()
print("RANK_OK", RANK)
"""


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_symmetric_memory_two_ranks_on_mock():
    port = _free_port()
    env = dict(os.environ, FOUNDRY_CUDA_DRIVER=MOCK, PYTHONPATH=ROOT, CUDA_VISIBLE_DEVICES="")
    procs = []
    for rank in range(2):
        code = f"ROOT={ROOT!r}; PORT={port}; RANK={rank}\n" + WORKER
        procs.append(subprocess.Popen([sys.executable, "-c", code], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.PIPE, text=True))
    outs = [p.communicate(timeout=180) for p in procs]
    for p, (o, e) in zip(procs, outs):
        assert p.returncode == 0, f"{o}\n{e}"
        assert "RANK_OK" in o
