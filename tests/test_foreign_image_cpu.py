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
