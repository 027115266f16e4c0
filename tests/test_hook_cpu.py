"""The interposer's driver entry points on the mock driver, called the way a
library would call them (ctypes on the preloaded libfoundry_hook.so):
cuMemAlloc_v2 / cuMemFree_v2 inside and outside the region, and
cuMemAddressReserve carving. Reservations below 2 GiB are carved from the
cursor and logged as Reserve events; larger ones are placed past the span;
freeing a carved range is a no-op that leaves the cursor where it is."""

import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "foundry_b200", "lib")

SCRIPT = r"""
import ctypes, json, sys
sys.path.insert(0, ROOT)
import foundry_b200 as fb
c = fb.core()
assert c.hook_is_preloaded() and c.driver_is_mock()
cu = ctypes.CDLL(None)
U64 = ctypes.c_uint64
for name, args in (("cuMemAlloc_v2", [ctypes.POINTER(U64), ctypes.c_size_t]), ("cuMemFree_v2", [U64]),
                   ("cuMemAddressReserve", [ctypes.POINTER(U64), ctypes.c_size_t, ctypes.c_size_t, U64,
                                            ctypes.c_ulonglong]),
                   ("cuMemAddressFree", [U64, ctypes.c_size_t])):
    getattr(cu, name).argtypes = args
    getattr(cu, name).restype = ctypes.c_int

base, size = 0x6b0000000000, 8 << 30
c.set_allocation_region(base, size)
gran = c.region_granularity()

# cuMemAlloc_v2 from "a library": lands at the cursor, cursor moves forward
p = U64(0)
assert cu.cuMemAlloc_v2(ctypes.byref(p), 3 << 20) == 0
assert base <= p.value < base + size, hex(p.value)
off1 = fb.get_current_alloc_offset()
assert off1 >= (3 << 20) and off1 % gran == 0
ctypes.memset(p.value, 7, 4096)                       # mock device memory is host memory
assert cu.cuMemFree_v2(p) == 0
assert fb.get_current_alloc_offset() == off1          # frees never rewind the cursor

# reservations: carved (< 2 GiB) and recorded
c.start_hook_record()
r = U64(0)
assert cu.cuMemAddressReserve(ctypes.byref(r), 64 << 20, 0, 0, 0) == 0
assert r.value == base + off1, (hex(r.value), hex(base + off1))
off2 = fb.get_current_alloc_offset()
assert off2 == off1 + (64 << 20)
c.end_hook_record()
ev = json.loads(c.hook_events_json())["events"]
assert [e["type"] for e in ev] == ["reserve"] and ev[0]["ptr"] == r.value and ev[0]["size"] == 64 << 20, ev
assert cu.cuMemAddressFree(r, 64 << 20) == 0          # carved: a no-op
assert fb.get_current_alloc_offset() == off2

# a large reservation (symmetric heaps, expandable segments) goes past the span
big = U64(0)
assert cu.cuMemAddressReserve(ctypes.byref(big), 4 << 30, 0, 0, 0) == 0
assert not (base <= big.value < base + size), hex(big.value)
assert fb.get_current_alloc_offset() == off2
assert cu.cuMemAddressFree(big, 4 << 30) == 0

# region stopped: allocations bypass it; resumed: back at the cursor
c.stop_allocation_region()
q = U64(0)
assert cu.cuMemAlloc_v2(ctypes.byref(q), 1 << 20) == 0
assert not (base <= q.value < base + size), hex(q.value)
assert cu.cuMemFree_v2(q) == 0
c.resume_allocation_region()
assert cu.cuMemAlloc_v2(ctypes.byref(q), 1 << 20) == 0
assert q.value == base + off2, (hex(q.value), hex(base + off2))

# pitched 2-D allocations land at the cursor; the pitch is the row width
# rounded up to the texture pitch alignment (mock: 32, raised to 128)
cu.cuMemAllocPitch_v2.argtypes = [ctypes.POINTER(U64), ctypes.POINTER(ctypes.c_size_t), ctypes.c_size_t,
                                  ctypes.c_size_t, ctypes.c_uint]
cu.cuMemAllocPitch_v2.restype = ctypes.c_int
off3 = fb.get_current_alloc_offset()
pp, pitch = U64(0), ctypes.c_size_t(0)
assert cu.cuMemAllocPitch_v2(ctypes.byref(pp), ctypes.byref(pitch), 1000, 64, 4) == 0
assert pitch.value == 1024 and pp.value == base + off3, (pitch.value, hex(pp.value))
ctypes.memset(pp.value + 63 * pitch.value, 1, 1000)  # the last row is mapped
assert fb.get_current_alloc_offset() > off3
assert cu.cuMemAllocPitch_v2(ctypes.byref(pp), ctypes.byref(pitch), 1000, 64, 3) != 0  # element size 3
print("HOOK_OK")
"""


def test_hook_entry_points_on_mock():
    env = dict(os.environ, FOUNDRY_CUDA_DRIVER=os.path.join(LIB, "libfoundry_mockcuda.so"), PYTHONPATH=ROOT,
               CUDA_VISIBLE_DEVICES="", LD_PRELOAD=os.path.join(LIB, "libfoundry_hook.so"))
    r = subprocess.run([sys.executable, "-c", f"ROOT={ROOT!r}\n" + SCRIPT], env=env, capture_output=True, text=True,
                       timeout=180)
    assert r.returncode == 0 and "HOOK_OK" in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]


FRONT_DOOR = r"""
import ctypes, sys
sys.path.insert(0, ROOT)
import foundry_b200 as fb
c = fb.core()
assert c.hook_is_preloaded() and c.driver_is_mock()
hook = ctypes.CDLL(HOOK)
addr = lambda f: ctypes.cast(f, ctypes.c_void_p).value
libdl = ctypes.CDLL(None)
libdl.dlopen.restype = ctypes.c_void_p
libdl.dlopen.argtypes = [ctypes.c_char_p, ctypes.c_int]
libdl.dlsym.restype = ctypes.c_void_p
libdl.dlsym.argtypes = [ctypes.c_void_p, ctypes.c_char_p]
drv = libdl.dlopen(MOCK.encode(), 2)  # RTLD_NOW, local: how a runtime opens the driver
assert drv
# dlsym on the driver handle: overridden entry points resolve to the interposer
for name in ("cuMemAlloc_v2", "cuMemFree_v2", "cuMemAllocPitch_v2", "cuMemAddressReserve", "cuLibraryLoadData",
             "cuIpcGetMemHandle"):
    assert libdl.dlsym(drv, name.encode()) == addr(getattr(hook, name)), name
# others stay the driver's, unknown names stay unknown
assert libdl.dlsym(drv, b"cuCtxGetDevice") == addr(ctypes.CDLL(MOCK).cuCtxGetDevice)
assert not libdl.dlsym(drv, b"cuNoSuchEntryPoint")
# cuGetProcAddress(base name, version) -> the versioned override
pfn = ctypes.c_void_p(0)
status = ctypes.c_int(0)
gpa = hook.cuGetProcAddress_v2
gpa.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, ctypes.c_uint64,
                ctypes.POINTER(ctypes.c_int)]
assert gpa(b"cuMemAlloc", ctypes.byref(pfn), 12080, 0, ctypes.byref(status)) == 0
assert pfn.value == addr(hook.cuMemAlloc_v2)
assert gpa(b"cuMemAlloc", ctypes.byref(pfn), 3000, 0, ctypes.byref(status)) == 0
assert pfn.value != addr(hook.cuMemAlloc_v2)          # pre-_v2 callers keep the driver's entry point
assert gpa(b"cuMemAllocPitch", ctypes.byref(pfn), 12080, 0, ctypes.byref(status)) == 0
assert pfn.value == addr(hook.cuMemAllocPitch_v2)
assert gpa(b"cuCtxGetDevice", ctypes.byref(pfn), 12080, 0, ctypes.byref(status)) == 0
assert pfn.value == addr(ctypes.CDLL(MOCK).cuCtxGetDevice)
print("FRONT_DOOR_OK")
"""


def test_symbol_front_door_on_mock():
    """dlsym and cuGetProcAddress route the overridden driver entry points to
    the interposer and leave every other symbol alone."""
    mock, hook = os.path.join(LIB, "libfoundry_mockcuda.so"), os.path.join(LIB, "libfoundry_hook.so")
    env = dict(os.environ, FOUNDRY_CUDA_DRIVER=mock, PYTHONPATH=ROOT, CUDA_VISIBLE_DEVICES="", LD_PRELOAD=hook)
    code = f"ROOT={ROOT!r}; MOCK={mock!r}; HOOK={hook!r}\n" + FRONT_DOOR
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=180)
    assert r.returncode == 0 and "FRONT_DOOR_OK" in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]
