"""Foreign code images on the mock driver. A shared library built here
embeds a code image and loads it through the interposed cuLibraryLoadData,
the way a vendor library loads its kernels. SAVE identifies the image by the
shared object that contains it and the offset from that object's load base,
and writes that reference. No byte of the image lands in the archive. A
fresh LOAD process re-opens the object, hands the driver the pointer at the
same offset, and resolves the kernel by (image hash, entry name)."""

import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "foundry_b200", "lib")
MARKER = "FOREIGN-IMAGE-MARKER-5f3a9c"

FAKE_LIB_C = r"""
#include <stddef.h>
typedef int CUresult;
typedef void* CUlibrary;
extern CUresult cuLibraryLoadData(CUlibrary* library, const void* code, void* jitOptions, void** jitOptionsValues,
                                  unsigned int numJitOptions, void* libraryOptions, void** libraryOptionValues,
                                  unsigned int numLibraryOptions);
/* mock image: header with the entry names and their parameter sizes, then payload */
static const char image[] = "FBMOCK\nfbfake_k:8,4\n\n" "@MARKER@" "....payload....";
int fake_load(CUlibrary* out) { return cuLibraryLoadData(out, image, NULL, NULL, 0, NULL, NULL, 0); }
"""

SAVE = r"""
import ctypes, json, os, sys
sys.path.insert(0, ROOT)
import foundry_b200 as fb
c = fb.core()
assert c.hook_is_preloaded() and c.driver_is_mock()
fake = ctypes.CDLL(FAKE)
lib = ctypes.c_void_p(0)
assert fake.fake_load(ctypes.byref(lib)) == 0 and lib.value
mock = ctypes.CDLL(MOCK)
k = ctypes.c_void_p(0)
mock.cuLibraryGetKernel.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p, ctypes.c_char_p]
assert mock.cuLibraryGetKernel(ctypes.byref(k), lib, b"fbfake_k") == 0 and k.value
h, name = c.identify_function(k.value)
assert name == "fbfake_k" and h != 0, (h, name)
c.mark_binary_used(h)
fb.pack_fatbins_to_folder(ARCH)
txt = open(os.path.join(ARCH, "fatbin_entrypoint_packed.txt")).read()
assert f"{h:016x}" in txt and "source=" + os.path.realpath(FAKE) in txt and "source_offset=" in txt, txt
img = open(os.path.join(ARCH, "fatbin_image_packed.img"), "rb").read()
assert MARKER.encode() not in img, "foreign image bytes were copied into the archive"
json.dump({"hash": h}, open(os.path.join(ARCH, "foreign.json"), "w"))
print("SAVE_OK")
"""

LOAD = r"""
import json, os, sys
sys.path.insert(0, ROOT)
import foundry_b200 as fb
c = fb.core()
assert c.hook_is_preloaded() and c.driver_is_mock()
h = json.load(open(os.path.join(ARCH, "foreign.json")))["hash"]
fb.set_skip_fatbin_processing(True)
fb.load_cuda_modules_and_libraries(ARCH)
f = c.query_function_handle(h, "fbfake_k")
assert f != 0
assert c.identify_function(f)[1] == "fbfake_k"
print("LOAD_OK")
"""


def test_foreign_image_by_object_and_offset(tmp_path):
    src = tmp_path / "fake.c"
    src.write_text(FAKE_LIB_C.replace("@MARKER@", MARKER))
    fake = str(tmp_path / "libfakekernels.so")
    subprocess.run(["gcc", "-shared", "-fPIC", "-O1", str(src), "-o", fake], check=True, timeout=120)
    arch = str(tmp_path / "arch")
    os.makedirs(arch)
    mock = os.path.join(LIB, "libfoundry_mockcuda.so")
    env = dict(os.environ, FOUNDRY_CUDA_DRIVER=mock, PYTHONPATH=ROOT, CUDA_VISIBLE_DEVICES="",
               LD_PRELOAD=os.path.join(LIB, "libfoundry_hook.so"))
    head = f"ROOT={ROOT!r}; FAKE={fake!r}; MOCK={mock!r}; ARCH={arch!r}; MARKER={MARKER!r}\n"
    for body, ok in ((SAVE, "SAVE_OK"), (LOAD, "LOAD_OK")):
        r = subprocess.run([sys.executable, "-c", head + body], env=env, capture_output=True, text=True, timeout=180)
        assert r.returncode == 0 and ok in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]


JIT_SAVE = r"""
import ctypes, json, os, sys
sys.path.insert(0, ROOT)
import foundry_b200 as fb
c = fb.core()
assert c.hook_is_preloaded() and c.driver_is_mock()
# an image compiled in this process (a JIT compiler's output), held on the heap
image = b"FBMOCK\nfbjit_k:8,4\n\n" + MARKER.encode() + bytes(range(256)) * 8
buf = ctypes.create_string_buffer(image, len(image))
drv = ctypes.CDLL(None)  # the preloaded interposer's cuModuleLoadData
mod = ctypes.c_void_p(0)
drv.cuModuleLoadData.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]
assert drv.cuModuleLoadData(ctypes.byref(mod), buf) == 0 and mod.value
fn = ctypes.c_void_p(0)
mock = ctypes.CDLL(MOCK)  # not interposed: straight to the driver
mock.cuModuleGetFunction.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p, ctypes.c_char_p]
assert mock.cuModuleGetFunction(ctypes.byref(fn), mod, b"fbjit_k") == 0 and fn.value
h_byname, name = c.identify_function(fn.value)  # heap image: only its entry name is known
assert name == "fbjit_k"
from foundry_b200 import jit
class K:  # the two attributes Triton's CompiledKernel carries
    module = mod.value
    kernel = image
h = jit.adopt_loaded_kernel(K)
assert h and h != h_byname
assert c.identify_function(fn.value) == (h, "fbjit_k")
c.mark_binary_used(h)
fb.pack_fatbins_to_folder(ARCH)
txt = open(os.path.join(ARCH, "fatbin_entrypoint_packed.txt")).read()
assert f"{h:016x}" in txt and "source=" not in txt, txt
img = open(os.path.join(ARCH, "fatbin_image_packed.img"), "rb").read()
assert image in img, "adopted image bytes missing from the pack"
json.dump({"hash": h}, open(os.path.join(ARCH, "jit.json"), "w"))
print("SAVE_OK")
"""

JIT_LOAD = r"""
import json, os, sys
sys.path.insert(0, ROOT)
import foundry_b200 as fb
c = fb.core()
h = json.load(open(os.path.join(ARCH, "jit.json")))["hash"]
fb.set_skip_fatbin_processing(True)
fb.load_cuda_modules_and_libraries(ARCH)
f = c.query_function_handle(h, "fbjit_k")
assert f != 0 and c.identify_function(f) == (h, "fbjit_k")
assert "triton" not in sys.modules  # nothing is recompiled on LOAD
print("LOAD_OK")
"""


def test_jit_compiled_image_is_packed_by_bytes(tmp_path):
    """A module loaded from heap bytes compiled in this process (Triton's
    case) is adopted with its exact bytes: the pack stores them and a fresh
    process reloads the kernel without the compiler."""
    arch = str(tmp_path / "arch")
    os.makedirs(arch)
    mock = os.path.join(LIB, "libfoundry_mockcuda.so")
    env = dict(os.environ, FOUNDRY_CUDA_DRIVER=mock, PYTHONPATH=ROOT, CUDA_VISIBLE_DEVICES="",
               LD_PRELOAD=os.path.join(LIB, "libfoundry_hook.so"))
    head = f"ROOT={ROOT!r}; ARCH={arch!r}; MARKER={MARKER!r}; MOCK={mock!r}\n"
    for script, ok in ((JIT_SAVE, "SAVE_OK"), (JIT_LOAD, "LOAD_OK")):
        r = subprocess.run([sys.executable, "-c", head + script], env=env, capture_output=True, text=True,
                           timeout=120)
        assert r.returncode == 0 and ok in r.stdout, r.stdout + r.stderr


NVSHMEM_VENDOR_C = r"""
typedef int CUresult;
typedef void* CUlibrary;
extern CUresult cuLibraryLoadData(CUlibrary* library, const void* code, void* jitOptions, void** jitOptionsValues,
                                  unsigned int numJitOptions, void* libraryOptions, void** libraryOptionValues,
                                  unsigned int numLibraryOptions);
/* a kernel image that references NVSHMEM's device state (like DeepEP's) */
static const char image[] = "FBMOCK\nfbep_dispatch:8,4\n@nvshmemi_device_state_d:64\n\n....payload....";
int vendor_load(CUlibrary* out) { return cuLibraryLoadData(out, image, 0, 0, 0, 0, 0, 0); }
"""

FAKE_NVSHMEM_C = r"""
static int calls = 0;
int nvshmemx_culibrary_init(void* lib) { (void)lib; ++calls; return 0; }
int nvshmemx_cumodule_init(void* mod) { (void)mod; ++calls; return 0; }
int fake_nvshmem_calls(void) { return calls; }
"""

NVSHMEM_SAVE = r"""
import ctypes, json, os, sys
sys.path.insert(0, ROOT)
import foundry_b200 as fb
c = fb.core()
vendor = ctypes.CDLL(VENDOR)
lib = ctypes.c_void_p(0)
assert vendor.vendor_load(ctypes.byref(lib)) == 0
mock = ctypes.CDLL(MOCK)
k = ctypes.c_void_p(0)
mock.cuLibraryGetKernel.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p, ctypes.c_char_p]
assert mock.cuLibraryGetKernel(ctypes.byref(k), lib, b"fbep_dispatch") == 0
h, _ = c.identify_function(k.value)
c.mark_binary_used(h)
fb.pack_fatbins_to_folder(ARCH)
lines = open(os.path.join(ARCH, "fatbin_entrypoint_packed.txt")).read().splitlines()
spec = lines[lines.index(f"{h:016x}") + 1]
assert spec.endswith(",binary_flags=2"), spec  # bit 1: needs NVSHMEM initialisation
json.dump({"hash": h}, open(os.path.join(ARCH, "nv.json"), "w"))
print("SAVE_OK")
"""

NVSHMEM_LOAD = r"""
import ctypes, json, os, sys
sys.path.insert(0, ROOT)
import foundry_b200 as fb
fb.set_nvshmem_auto_init(False)
fb.set_skip_fatbin_processing(True)
fb.load_cuda_modules_and_libraries(ARCH)
try:
    fb.init_nvshmem_for_loaded_modules()
    raise AssertionError("init succeeded without an NVSHMEM host library")
except RuntimeError as e:
    assert "NVSHMEM" in str(e), e
nv = ctypes.CDLL(NVSHMEM, mode=ctypes.RTLD_GLOBAL)  # the process's NVSHMEM host library
assert fb.init_nvshmem_for_loaded_modules() == 1
assert nv.fake_nvshmem_calls() == 1
assert fb.init_nvshmem_for_loaded_modules() == 0  # flushed: nothing pending
print("LOAD_OK")
"""


def test_nvshmem_images_flagged_and_initialised_on_load(tmp_path):
    """An image carrying NVSHMEM's device symbols is flagged in the pack
    (binary_flags bit 1); LOAD queues it and init_nvshmem_for_loaded_modules
    hands it to the process's NVSHMEM host library exactly once."""
    libs = {}
    for name, src in (("vendor", NVSHMEM_VENDOR_C), ("nvshmem", FAKE_NVSHMEM_C)):
        c = tmp_path / f"{name}.c"
        c.write_text(src)
        libs[name] = str(tmp_path / f"lib{name}.so")
        subprocess.run(["gcc", "-shared", "-fPIC", "-O1", str(c), "-o", libs[name]], check=True, timeout=120)
    arch = str(tmp_path / "arch")
    os.makedirs(arch)
    mock = os.path.join(LIB, "libfoundry_mockcuda.so")
    env = dict(os.environ, FOUNDRY_CUDA_DRIVER=mock, PYTHONPATH=ROOT, CUDA_VISIBLE_DEVICES="",
               LD_PRELOAD=os.path.join(LIB, "libfoundry_hook.so"))
    head = (f"ROOT={ROOT!r}; ARCH={arch!r}; MOCK={mock!r}; VENDOR={libs['vendor']!r}; "
            f"NVSHMEM={libs['nvshmem']!r}\n")
    for script, ok in ((NVSHMEM_SAVE, "SAVE_OK"), (NVSHMEM_LOAD, "LOAD_OK")):
        r = subprocess.run([sys.executable, "-c", head + script], env=env, capture_output=True, text=True,
                           timeout=120)
        assert r.returncode == 0 and ok in r.stdout, r.stdout + r.stderr


OPTIONS_VENDOR_C = r"""
#include <stddef.h>
#include <stdint.h>
typedef int CUresult;
typedef void* CUmodule;
typedef void* CUlibrary;
extern CUresult cuModuleLoadDataEx(CUmodule* m, const void* image, unsigned int n, int* options, void** values);
extern CUresult cuLibraryLoadData(CUlibrary* library, const void* code, int* jitOptions, void** jitOptionsValues,
                                  unsigned int numJitOptions, int* libraryOptions, void** libraryOptionValues,
                                  unsigned int numLibraryOptions);
static const char image_a[] = "FBMOCK\nfbopt_a:8\n\n....a....";
static const char image_b[] = "FBMOCK\nfbopt_b:8\n\n....b....";
static char log_buf[1024];
int vendor_load(CUmodule* m, CUlibrary* l) {
  /* CU_JIT_MAX_REGISTERS=0 (64), CU_JIT_INFO_LOG_BUFFER=3 (a pointer: not kept),
     CU_JIT_INFO_LOG_BUFFER_SIZE_BYTES=4 (not kept), CU_JIT_OPTIMIZATION_LEVEL=7 (3) */
  int o[4] = {0, 3, 4, 7};
  void* v[4] = {(void*)(uintptr_t)64, log_buf, (void*)(uintptr_t)sizeof(log_buf), (void*)(uintptr_t)3};
  CUresult rc = cuModuleLoadDataEx(m, image_a, 4, o, v);
  if (rc) return rc;
  /* CU_JIT_MAX_REGISTERS=32; library option CU_LIBRARY_BINARY_IS_PRESERVED=1 (1) */
  int jo[1] = {0};
  void* jv[1] = {(void*)(uintptr_t)32};
  int lo[1] = {1};
  void* lv[1] = {(void*)(uintptr_t)1};
  return cuLibraryLoadData(l, image_b, jo, jv, 1, lo, lv, 1);
}
"""

OPTIONS_SAVE = r"""
import ctypes, json, os, sys
sys.path.insert(0, ROOT)
import foundry_b200 as fb
c = fb.core()
vendor = ctypes.CDLL(VENDOR)
m, l = ctypes.c_void_p(0), ctypes.c_void_p(0)
assert vendor.vendor_load(ctypes.byref(m), ctypes.byref(l)) == 0
mock = ctypes.CDLL(MOCK)
mock.cuModuleGetFunction.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p, ctypes.c_char_p]
mock.cuLibraryGetKernel.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p, ctypes.c_char_p]
fa, kb = ctypes.c_void_p(0), ctypes.c_void_p(0)
assert mock.cuModuleGetFunction(ctypes.byref(fa), m, b"fbopt_a") == 0
assert mock.cuLibraryGetKernel(ctypes.byref(kb), l, b"fbopt_b") == 0
for f in (fa, kb):
    c.mark_binary_used(c.identify_function(f.value)[0])
fb.pack_fatbins_to_folder(ARCH)
txt = open(os.path.join(ARCH, "fatbin_entrypoint_packed.txt")).read()
assert "cuModuleLoadDataEx,jit0=64,jit7=3,source=" in txt, txt
assert "cuLibraryLoadData,jit0=32,libopt1=1,source=" in txt, txt
print("SAVE_OK")
"""

OPTIONS_LOAD = r"""
import ctypes, os, sys
sys.path.insert(0, ROOT)
import foundry_b200 as fb
fb.set_skip_fatbin_processing(True)
fb.load_cuda_modules_and_libraries(ARCH)
mock = ctypes.CDLL(MOCK)
buf = ctypes.create_string_buffer(512)
log = []
while mock.fbmock_load_log(len(log), buf, 512) >= 0:
    log.append(buf.value.decode())
assert "cuModuleLoadDataEx jit0=64 jit7=3" in log, log
assert "cuLibraryLoadData jit0=32 lib1=1" in log, log
print("LOAD_OK")
"""


def test_foreign_load_options_are_replayed(tmp_path):
    """Scalar JIT / library options of a foreign image's load are written to
    the pack and passed to the same loader on LOAD; pointer and output
    options (log buffers) are not kept."""
    src = tmp_path / "vendor.c"
    src.write_text(OPTIONS_VENDOR_C)
    vendor = str(tmp_path / "libvendoropts.so")
    subprocess.run(["gcc", "-shared", "-fPIC", "-O1", str(src), "-o", vendor], check=True, timeout=120)
    arch = str(tmp_path / "arch")
    os.makedirs(arch)
    mock = os.path.join(LIB, "libfoundry_mockcuda.so")
    env = dict(os.environ, FOUNDRY_CUDA_DRIVER=mock, PYTHONPATH=ROOT, CUDA_VISIBLE_DEVICES="",
               LD_PRELOAD=os.path.join(LIB, "libfoundry_hook.so"))
    head = f"ROOT={ROOT!r}; ARCH={arch!r}; MOCK={mock!r}; VENDOR={vendor!r}\n"
    for script, ok in ((OPTIONS_SAVE, "SAVE_OK"), (OPTIONS_LOAD, "LOAD_OK")):
        r = subprocess.run([sys.executable, "-c", head + script], env=env, capture_output=True, text=True,
                           timeout=120)
        assert r.returncode == 0 and ok in r.stdout, r.stdout + r.stderr


LAZY_SAVE = r"""
import ctypes, json, os, sys
sys.path.insert(0, ROOT)
import foundry_b200 as fb
c = fb.core()
# a library that loads its kernels on first use, from heap memory (cuBLAS does)
image = b"FBMOCK\nfblazy_k:8,4\n\n" + bytes(64)
buf = ctypes.create_string_buffer(image, len(image))
drv = ctypes.CDLL(None)
mod = ctypes.c_void_p(0)
drv.cuModuleLoadData.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]
assert drv.cuModuleLoadData(ctypes.byref(mod), buf) == 0
mock = ctypes.CDLL(MOCK)
mock.cuModuleGetFunction.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p, ctypes.c_char_p]
fn = ctypes.c_void_p(0)
assert mock.cuModuleGetFunction(ctypes.byref(fn), mod, b"fblazy_k") == 0
h, name = c.identify_function(fn.value)
c.mark_binary_used(h)
fb.pack_fatbins_to_folder(ARCH)
c.set_allocation_region(0x600000000000, 1 << 30)
p = c.region_alloc(1 << 20)
prm = [{"index": 0, "offset": 0, "size": 8, "value_hex": p.to_bytes(8, "little").hex()},
       {"index": 1, "offset": 8, "size": 4, "value_hex": "07000000"}]
node = {"id": 0, "type": "KernelNode", "params": {"blockDimX": 32, "blockDimY": 1, "blockDimZ": 1, "gridDimX": 1,
        "gridDimY": 1, "gridDimZ": 1, "sharedMemBytes": 0, "kernelParams": prm, "function_name": name,
        "kernel_source_binary_hash": f"{h:016x}"}}
d = c.graph_from_json_text(json.dumps({"nodes": [node], "dependencies": [], "topology_key": "", "generators": [],
                                       "num_events": 0}))
c.recompute_topology_key(d)
d.save(os.path.join(ARCH, "graph_0.json"))
print("SAVE_OK")
"""

LAZY_LOAD = r"""
import ctypes, os, sys
sys.path.insert(0, ROOT)
import foundry_b200 as fb
c = fb.core()
fb.set_skip_fatbin_processing(True)
fb.load_cuda_modules_and_libraries(ARCH)
c.set_allocation_region(0x600000000000, 1 << 30)
c.region_alloc(1 << 20)
path = os.path.join(ARCH, "graph_0.json")
pending = c.start_graph_builds([path], 1)  # the library has not loaded its kernel yet
pending.wait()                             # background builds defer the graph instead of failing
if LOAD_LIBRARY:
    image = b"FBMOCK\nfblazy_k:8,4\n\n" + bytes(64)
    buf = ctypes.create_string_buffer(image, len(image))
    drv = ctypes.CDLL(None)
    mod = ctypes.c_void_p(0)
    drv.cuModuleLoadData.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]
    assert drv.cuModuleLoadData(ctypes.byref(mod), buf) == 0
    g = pending.finish_one(0)
    g.launch(0)
    print("LOAD_OK")
else:
    try:
        pending.finish_one(0)
        raise AssertionError("resolved a kernel no library loaded")
    except RuntimeError as e:
        assert "persisted by name" in str(e), e
    print("LOAD_REFUSED_OK")
"""


def test_by_name_kernels_resolve_when_the_graph_is_finished(tmp_path):
    """A graph whose kernel a library loads lazily (persisted by entry name)
    restores when its library has loaded the kernel by finish time, even if
    the background builds started earlier; without it, finish_one fails with
    a clear message."""
    arch = str(tmp_path / "arch")
    os.makedirs(arch)
    mock = os.path.join(LIB, "libfoundry_mockcuda.so")
    env = dict(os.environ, FOUNDRY_CUDA_DRIVER=mock, PYTHONPATH=ROOT, CUDA_VISIBLE_DEVICES="",
               LD_PRELOAD=os.path.join(LIB, "libfoundry_hook.so"))
    head = f"ROOT={ROOT!r}; ARCH={arch!r}; MOCK={mock!r}\n"
    runs = ((LAZY_SAVE, "SAVE_OK", ""), (LAZY_LOAD, "LOAD_OK", "LOAD_LIBRARY = True\n"),
            (LAZY_LOAD, "LOAD_REFUSED_OK", "LOAD_LIBRARY = False\n"))
    for script, ok, extra in runs:
        r = subprocess.run([sys.executable, "-c", head + extra + script], env=env, capture_output=True, text=True,
                           timeout=120)
        assert r.returncode == 0 and ok in r.stdout, r.stdout + r.stderr
