"""CUDA IPC on region memory (csrc/hook/ipc.cpp) on the mock driver, across
two processes: the exporter's cuIpcGetMemHandle on a region chunk yields a
handle that carries its pid and the allocation's POSIX fd. The importer (its
parent) duplicates the fd with pidfd_getfd and maps the allocation at the
exporter's address: the same pointer value reads the exporter's bytes.
A second open of the same chunk is reference-counted; close unmaps."""

import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "foundry_b200", "lib")
MOCK = os.path.join(LIB, "libfoundry_mockcuda.so")
HOOK = os.path.join(LIB, "libfoundry_hook.so")

EXPORTER = r"""
import ctypes, sys
sys.path.insert(0, ROOT)
import foundry_b200 as fb
c = fb.core()
assert c.hook_is_preloaded() and c.driver_is_mock()
c.set_allocation_region(0x6a0000000000, 1 << 30)
p = c.region_alloc(4 << 20)
ctypes.memmove(p + 4096, b"foundry-ipc-" + bytes(range(52)), 64)
lib = ctypes.CDLL(None)
handle = (ctypes.c_ubyte * 64)()
rc = lib.cuIpcGetMemHandle(handle, ctypes.c_uint64(p + 4096))
assert rc == 0, rc
print(hex(p + 4096), bytes(handle).hex(), flush=True)
sys.stdin.readline()   # stay alive (and keep the fd) until the importer is done
print("EXPORTER_DONE", flush=True)
"""

IMPORTER = r"""
import ctypes, os, subprocess, sys
sys.path.insert(0, ROOT)
import foundry_b200 as fb
c = fb.core()
assert c.hook_is_preloaded() and c.driver_is_mock()
child = subprocess.Popen([sys.executable, "-c", f"ROOT={ROOT!r}\n" + EXPORTER], stdin=subprocess.PIPE, stdout=subprocess.PIPE,
                         text=True, env=os.environ)
ptr_hex, handle_hex = child.stdout.readline().split()
ptr = int(ptr_hex, 16)
lib = ctypes.CDLL(None)


class IpcHandle(ctypes.Structure):  # CUipcMemHandle: 64 bytes, passed by value
    _fields_ = [("reserved", ctypes.c_ubyte * 64)]


handle = IpcHandle.from_buffer_copy(bytes.fromhex(handle_hex))
lib.cuIpcOpenMemHandle_v2.argtypes = [ctypes.POINTER(ctypes.c_uint64), IpcHandle, ctypes.c_uint]
out = ctypes.c_uint64(0)
rc = lib.cuIpcOpenMemHandle_v2(ctypes.byref(out), handle, 1)
assert rc == 0, rc
assert out.value == ptr, (hex(out.value), hex(ptr))           # same pointer value as in the exporter
assert ctypes.string_at(out.value, 64) == b"foundry-ipc-" + bytes(range(52))
out2 = ctypes.c_uint64(0)
assert lib.cuIpcOpenMemHandle_v2(ctypes.byref(out2), handle, 1) == 0 and out2.value == ptr  # ref-counted
lib.cuIpcCloseMemHandle.argtypes = [ctypes.c_uint64]
assert lib.cuIpcCloseMemHandle(ptr) == 0
assert lib.cuIpcCloseMemHandle(ptr) == 0
child.stdin.write("done\n"); child.stdin.flush()
assert "EXPORTER_DONE" in child.stdout.readline()
child.wait(timeout=60)
print("IPC_OK")
"""


def test_region_ipc_across_processes():
    env = dict(os.environ, FOUNDRY_CUDA_DRIVER=MOCK, PYTHONPATH=ROOT, CUDA_VISIBLE_DEVICES="", LD_PRELOAD=HOOK)
    code = f"ROOT={ROOT!r}\nEXPORTER={EXPORTER!r}\n" + IMPORTER
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=180)
    assert r.returncode == 0 and "IPC_OK" in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]
