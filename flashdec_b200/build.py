"""Build libflashdec_b200.so (the C-ABI + sm_100a kernels) in-tree with nvcc,
and the C++ host-path module ``_hostpath`` (csrc/fd_hostpath.cpp) with g++
against the installed torch.

    python -m flashdec_b200.build          # or: python flashdec_b200/build.py

Both land next to this file so that they travel with the source tree.
Objects are compiled in parallel and re-used when their sources are older.
"""

from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = REPO / "include"
BUILD = PKG / "_build"
LIB = PKG / "libflashdec_b200.so"
SOURCES = ["fd_host.cu", "fd_attention.cu", "fd_wave_decode.cu", "fd_rope_append.cu", "fd_static.cu", "fd_selftest.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
         "-I", str(INCLUDE), "-I", str(CSRC)]


def nvcc() -> str:
    cand = shutil.which("nvcc")
    if cand:
        return cand
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = Path(home) / "bin" / "nvcc"
    if path.exists():
        return str(path)
    raise RuntimeError("nvcc not found (set CUDA_HOME)")


def _deps_mtime() -> float:
    files = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max(f.stat().st_mtime for f in files)


def _compile(src: str, verbose: bool) -> Path:
    obj = BUILD / (Path(src).stem + ".o")
    s = CSRC / src
    if obj.exists() and obj.stat().st_mtime >= max(s.stat().st_mtime, _deps_mtime()):
        return obj
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(s), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr:
        print(res.stderr, flush=True)
    return obj


HOSTPATH_SRC = CSRC / "fd_hostpath.cpp"
HOSTPATH = PKG / ("_hostpath" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_hostpath(verbose: bool = False, force: bool = False) -> Path:
    """Compile the torch extension module of the C++ host path with g++
    (no JIT: the module is a plain in-tree file, loaded like the library)."""
    import torch
    from torch.utils import cpp_extension

    newest = max(HOSTPATH_SRC.stat().st_mtime, (INCLUDE / "flashdec_b200.h").stat().st_mtime)
    if HOSTPATH.exists() and HOSTPATH.stat().st_mtime >= newest and not force:
        return HOSTPATH
    incs = cpp_extension.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"],
                                                              str(INCLUDE)]
    libs = cpp_extension.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    tmp = HOSTPATH.with_suffix(".tmp")
    cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-shared", "-fPIC",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_hostpath",
           "-DTORCH_API_INCLUDE_EXTENSION_H", *[f"-I{d}" for d in incs],
           str(HOSTPATH_SRC), "-o", str(tmp), *[f"-L{d}" for d in libs],
           "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lcudart",
           *[f"-Wl,-rpath,{d}" for d in libs]]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"g++ failed for {HOSTPATH_SRC.name}:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, HOSTPATH)
    return HOSTPATH


def build(verbose: bool = False, force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    with concurrent.futures.ThreadPoolExecutor(max_workers=1) as hp:
        hostpath = hp.submit(build_hostpath, verbose, force)
        lib = _build_library(verbose, force)
        hostpath.result()
    return lib


def _build_library(verbose: bool, force: bool) -> Path:
    if force:
        for o in BUILD.glob("*.o"):
            o.unlink()
    with concurrent.futures.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), SOURCES))
    newest = max(o.stat().st_mtime for o in objs)
    if LIB.exists() and LIB.stat().st_mtime >= newest and not force:
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp), *map(str, objs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
