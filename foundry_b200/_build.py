"""Native build driver for foundry_b200.

Builds, in-tree (so the artefacts travel with the source tree):

* ``foundry_b200/lib/libfoundry_hook.so``   the LD_PRELOAD interposer, VMM region,
  event log and module registry (C++17, no CUDA link: the driver is dlopen'ed);
* ``foundry_b200/lib/libfoundry_mockcuda.so`` the CPU-only mock driver for tests;
* ``foundry_b200/_C*.so``                    pybind11 module: graph core + kernel runtime;
* ``foundry_b200/kernels/*.cubin``           sm_100a kernels (``nvcc -cubin
  -gencode arch=compute_100a,code=sm_100a``), loaded at run time through the
  module registry so every kernel in a persisted graph has a content hash.

Rebuilds only what changed (a stamp holds the hash of sources + flags).
Parity: reference CMakeLists.txt:1-45 and setup.py:14-142 (CMake + setuptools
with Boost); ours is a dependency-free Python driver around g++ and nvcc.
"""

from __future__ import annotations

import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "foundry_b200"
CSRC = ROOT / "csrc"
LIB = PKG / "lib"
KDIR = PKG / "kernels"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

CXXFLAGS = [
    "-std=c++17", "-O2", "-fPIC", "-Wall", "-Wno-unused-parameter",
    "-Wno-maybe-uninitialized", f"-I{CUDA_HOME / 'include'}",
]
NVCCFLAGS = [
    "-std=c++17", "-O3", "-lineinfo", "--use_fast_math", "-Xptxas=-v",
    "--expt-relaxed-constexpr", f"-I{CSRC / 'kernels'}",
] + ARCH


def _digest(paths, extra: str) -> str:
    h = hashlib.sha256(extra.encode())
    for p in sorted(paths):
        h.update(str(p).encode())
        h.update(Path(p).read_bytes())
    return h.hexdigest()


def _up_to_date(out: Path, digest: str) -> bool:
    stamp = out.with_name(out.name + ".stamp")
    return out.exists() and stamp.exists() and stamp.read_text() == digest


def _stamp(out: Path, digest: str) -> None:
    out.with_name(out.name + ".stamp").write_text(digest)


def _run(cmd, log=None) -> str:
    res = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(cmd)}\n{res.stdout}")
    return res.stdout


def ext_suffix() -> str:
    return sysconfig.get_config_var("EXT_SUFFIX") or ".so"


def build_hook(force=False) -> Path:
    out = LIB / "libfoundry_hook.so"
    srcs = sorted((CSRC / "hook").glob("*.cpp"))
    deps = srcs + sorted((CSRC / "hook").glob("*.h")) + sorted((CSRC / "common").glob("*.h"))
    d = _digest(deps, " ".join(CXXFLAGS))
    if not force and _up_to_date(out, d):
        return out
    LIB.mkdir(parents=True, exist_ok=True)
    tmp = out.with_suffix(".so.tmp")
    _run(["g++", *CXXFLAGS, "-shared", *map(str, srcs), "-o", str(tmp), "-ldl", "-lpthread"])
    os.replace(tmp, out)
    _stamp(out, d)
    return out


def build_mock(force=False) -> Path:
    out = LIB / "libfoundry_mockcuda.so"
    srcs = [CSRC / "mockcuda" / "mock_cuda.cpp"]
    d = _digest(srcs, " ".join(CXXFLAGS))
    if not force and _up_to_date(out, d):
        return out
    LIB.mkdir(parents=True, exist_ok=True)
    tmp = out.with_suffix(".so.tmp")
    _run(["g++", *CXXFLAGS, "-shared", *map(str, srcs), "-o", str(tmp), "-ldl", "-lpthread"])
    os.replace(tmp, out)
    _stamp(out, d)
    return out


def build_core(force=False) -> Path:
    import pybind11

    out = PKG / f"_C{ext_suffix()}"
    srcs = sorted((CSRC / "core").glob("*.cpp"))
    deps = srcs + sorted((CSRC / "core").glob("*.h")) + sorted((CSRC / "common").glob("*.h"))
    inc = [f"-I{sysconfig.get_paths()['include']}", f"-I{pybind11.get_include()}"]
    d = _digest(deps, " ".join(CXXFLAGS + inc))
    if not force and _up_to_date(out, d) and (LIB / "libfoundry_hook.so").exists():
        return out
    objdir = ROOT / "build" / "core"
    objdir.mkdir(parents=True, exist_ok=True)

    def compile_one(src: Path) -> Path:
        obj = objdir / (src.stem + ".o")
        _run(["g++", *CXXFLAGS, *inc, "-c", str(src), "-o", str(obj)])
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(compile_one, srcs))
    tmp = out.with_name(out.name + ".tmp")
    _run(["g++", "-shared", *map(str, objs), "-o", str(tmp), f"-L{LIB}", "-lfoundry_hook",
          "-Wl,-rpath,$ORIGIN/lib", "-ldl", "-lpthread"])
    os.replace(tmp, out)
    _stamp(out, d)
    return out


def build_torchrng(force=False) -> Path:
    """``foundry_b200/_torchrng*.so``: reads the graph-capture state of torch's
    default CUDA generators (links libtorch; loaded only when a graph that
    draws random numbers is saved or restored)."""
    import torch

    tdir = Path(torch.__file__).resolve().parent
    out = PKG / f"_torchrng{ext_suffix()}"
    src = CSRC / "torchrng" / "rng_state.cpp"
    abi = int(bool(torch._C._GLIBCXX_USE_CXX11_ABI))
    inc = [f"-I{sysconfig.get_paths()['include']}", f"-I{tdir / 'include'}",
           f"-I{tdir / 'include' / 'torch' / 'csrc' / 'api' / 'include'}", f"-I{CUDA_HOME / 'include'}"]
    flags = ["-std=c++17", "-O2", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_torchrng",
             "-w"]
    d = _digest([src], " ".join(flags + inc + [torch.__version__]))
    if not force and _up_to_date(out, d):
        return out
    tmp = out.with_name(out.name + ".tmp")
    _run(["g++", *flags, *inc, "-shared", str(src), "-o", str(tmp), f"-L{tdir / 'lib'}", "-lc10", "-lc10_cuda",
          "-ltorch_cpu", "-ltorch_cuda", f"-Wl,-rpath,{tdir / 'lib'}"])
    os.replace(tmp, out)
    _stamp(out, d)
    return out


def kernel_sources():
    return sorted((CSRC / "kernels").glob("*.cu"))


def build_kernel(src: Path, force=False) -> tuple[Path, str]:
    out = KDIR / (src.stem + ".cubin")
    headers = sorted((CSRC / "kernels").glob("*.cuh"))
    d = _digest([src, *headers], " ".join(NVCCFLAGS))
    if not force and _up_to_date(out, d):
        return out, ""
    KDIR.mkdir(parents=True, exist_ok=True)
    tmp = out.with_suffix(".cubin.tmp")
    log = _run([NVCC, *NVCCFLAGS, "-cubin", str(src), "-o", str(tmp)])
    os.replace(tmp, out)
    _stamp(out, d)
    (KDIR / (src.stem + ".ptxas.txt")).write_text(log)
    return out, log


def build_kernels(force=False, jobs=None) -> list[Path]:
    srcs = kernel_sources()
    jobs = jobs or min(8, os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        res = list(ex.map(lambda s: build_kernel(s, force), srcs))
    return [r[0] for r in res]


def build_noalloc(force=False) -> Path:
    """``lib/libfoundry_noalloc.so``: the decode-attention entry point with a
    static scratch buffer (runtime API, static cudart, one exported symbol)."""
    out = LIB / "libfoundry_noalloc.so"
    src = CSRC / "noalloc" / "decode_attn_noalloc.cu"
    headers = [CSRC / "noalloc" / "decode_attn_noalloc.h", CSRC / "kernels" / "attention.cu",
               *sorted((CSRC / "kernels").glob("*.cuh"))]
    flags = [f for f in NVCCFLAGS if f != "-Xptxas=-v"] + ["-rdc=true", "-shared", "-Xcompiler", "-fPIC,-fvisibility=hidden"]
    d = _digest([src, *headers], " ".join(flags))
    if not force and _up_to_date(out, d):
        return out
    LIB.mkdir(parents=True, exist_ok=True)
    tmp = out.with_suffix(".so.tmp")
    _run([NVCC, *flags, str(src), "-o", str(tmp)])
    os.replace(tmp, out)
    _stamp(out, d)
    return out


def build_tsan(dest: Path) -> Path:
    """ThreadSanitizer build of the host libraries (hook, mock driver, _C) in a
    copy of the Python package under ``dest`` (race detection of the region,
    registry and parallel-restore threads on the mock driver; run the copy
    with LD_PRELOAD of libtsan). Returns the folder to put on PYTHONPATH."""
    import pybind11

    dest = Path(dest)
    pkg = dest / "foundry_b200"
    if pkg.exists():
        shutil.rmtree(pkg)
    shutil.copytree(PKG, pkg, ignore=shutil.ignore_patterns("*.so", "*.stamp", "__pycache__", "kernels", "*.tmp"))
    (pkg / "lib").mkdir(exist_ok=True)
    tsan = ["-fsanitize=thread", "-g", "-O1", "-fno-omit-frame-pointer"]
    flags = [f for f in CXXFLAGS if f != "-O2"] + tsan
    hook_srcs = sorted((CSRC / "hook").glob("*.cpp"))
    _run(["g++", *flags, "-shared", *map(str, hook_srcs), "-o", str(pkg / "lib" / "libfoundry_hook.so"), "-ldl",
          "-lpthread"])
    _run(["g++", *flags, "-shared", str(CSRC / "mockcuda" / "mock_cuda.cpp"), "-o",
          str(pkg / "lib" / "libfoundry_mockcuda.so"), "-ldl", "-lpthread"])
    inc = [f"-I{sysconfig.get_paths()['include']}", f"-I{pybind11.get_include()}"]
    objdir = dest / "obj"
    objdir.mkdir(parents=True, exist_ok=True)

    def compile_one(src: Path) -> Path:
        obj = objdir / (src.stem + ".o")
        _run(["g++", *flags, *inc, "-c", str(src), "-o", str(obj)])
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(compile_one, sorted((CSRC / "core").glob("*.cpp"))))
    _run(["g++", *tsan, "-shared", *map(str, objs), "-o", str(pkg / f"_C{ext_suffix()}"), f"-L{pkg / 'lib'}",
          "-lfoundry_hook", "-Wl,-rpath,$ORIGIN/lib", "-ldl", "-lpthread"])
    return dest


def build_all(force=False, kernels=True) -> None:
    build_hook(force)
    build_mock(force)
    build_core(force)
    build_torchrng(force)
    if kernels:
        if shutil.which(NVCC) is None and not Path(NVCC).exists():
            raise RuntimeError(f"nvcc not found at {NVCC}")
        build_kernels(force)
        build_noalloc(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, kernels="--no-kernels" not in sys.argv)
    print("foundry_b200 native build complete")
