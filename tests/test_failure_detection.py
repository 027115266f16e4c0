"""Failure detection without faulting a GPU.

* host side (CPU, gloo ranks on the mock driver): a rank that never joins the
  symmetric-memory handle exchange ends the others with an error, not a hang;
* device side (one GPU): a barrier whose peer never arrives (a flag nothing
  sets) gives up after its bounded wait, records FB_KERR_TIMEOUT_PEER in the
  image's status word and returns; the context stays usable.
"""

import os
import socket
import subprocess
import sys
import time

import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
MOCK = os.path.join(ROOT, "foundry_b200", "lib", "libfoundry_mockcuda.so")

WORKER = r"""
import os, sys, time
import torch.distributed as dist
from datetime import timedelta
sys.path.insert(0, ROOT)
dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % PORT, rank=RANK, world_size=2,
                        timeout=timedelta(seconds=20))
if RANK == 1:
    os._exit(0)  # dies before the exchange
from foundry_b200.parallel.symm import SymmetricMemory
c = __import__("foundry_b200").core()
c.set_allocation_region(0x600000000000, 1 << 30)
t0 = time.time()
try:
    SymmetricMemory(8 << 20, multicast=False)
except Exception as e:  # noqa: BLE001
    print("FAILED_AS_EXPECTED", type(e).__name__, round(time.time() - t0, 1))
    sys.exit(0)
print("UNEXPECTED_SUCCESS")
sys.exit(1)
"""


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_rank_that_never_joins_ends_the_exchange_with_an_error():
    port = _free_port()
    env = dict(os.environ, FOUNDRY_CUDA_DRIVER=MOCK, PYTHONPATH=ROOT, CUDA_VISIBLE_DEVICES="")
    procs = [subprocess.Popen([sys.executable, "-c", f"ROOT={ROOT!r}; PORT={port}; RANK={r}\n" + WORKER], env=env,
                              stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True) for r in range(2)]
    t0 = time.time()
    out0, err0 = procs[0].communicate(timeout=180)
    procs[1].communicate(timeout=60)
    assert procs[0].returncode == 0, f"{out0}\n{err0[-3000:]}"
    assert "FAILED_AS_EXPECTED" in out0
    assert time.time() - t0 < 150


@pytest.mark.gpu
def test_barrier_wait_times_out_and_reports_status():
    from foundry_b200 import core, ops
    from foundry_b200.ops import _rt

    c = core()
    dev = torch.cuda.current_device()
    gran = c.vmm_granularity(dev)
    size = gran
    base = 0x780000000000
    h0, h1 = c.vmm_create(size, dev), c.vmm_create(size, dev)
    va = c.vmm_reserve(base, 2 * size, gran)
    try:
        c.vmm_map(base, size, h0, 0)
        c.vmm_map(base + size, size, h1, 0)
        c.vmm_set_access(base, 2 * size, [dev])
        from foundry_b200.graphs import tensor_from_ptr

        tensor_from_ptr(base, (2 * size,), (1,), torch.uint8).zero_()
        _rt.clear_status("comm")
        torch.cuda.synchronize()
        t0 = time.time()
        # rank 0 of a 2-rank barrier whose rank 1 never arrives
        _rt.launch("comm", "fb_sym_barrier", (1,), (64,), [base, size, 0, 2])
        torch.cuda.synchronize()
        waited = time.time() - t0
        assert ops.status("comm") & 8, ops.status("comm")  # FB_KERR_TIMEOUT_PEER
        assert 1.0 < waited < 30.0, waited
        # the context is still usable: a 1-rank barrier and a tensor op complete
        _rt.clear_status("comm")
        _rt.launch("comm", "fb_sym_barrier", (1,), (64,), [base, size, 0, 1])
        x = torch.ones(1024, device="cuda").sum()
        torch.cuda.synchronize()
        assert ops.status("comm") == 0 and int(x.item()) == 1024
    finally:
        torch.cuda.synchronize()
        c.vmm_unmap(base, size)
        c.vmm_unmap(base + size, size)
        c.vmm_release(h0)
        c.vmm_release(h1)
        c.vmm_free_va(va, 2 * size)
