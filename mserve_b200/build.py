"""Builds libmserve_kv.so (the sm_100a CUDA library behind the C ABI in include/mserve_kv.h).

Usage: ``python -m mserve_b200.build`` (or ``__graft_entry__.build()``).  Every ``.cu`` file
under ``mserve_b200/csrc`` is compiled by nvcc for ``sm_100a`` only and linked into
``mserve_b200/libmserve_kv.so``; objects go to ``_build/``.  The library is rebuilt only when
a source or header is newer than it.

``build_torch_ext()`` then builds the ``cuda_uva`` torch extension
(``mserve_b200/torch_ext/cuda_uva.cpp``, pybind11 + ATen, no device code of its own) into
``mserve_b200/torch_ext/``, linked against ``libmserve_kv.so`` beside it: with that directory on
``sys.path`` an unmodified ``import cuda_uva`` resolves to this library.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build" / "mserve_kv"
LIB = PKG / "libmserve_kv.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
              "--expt-relaxed-constexpr", f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libmserve_kv.so")
    return cand


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _deps():
    return _sources() + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h")) + [Path(__file__)]


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _deps())


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compiles and links the library; returns its path."""
    if not force and up_to_date():
        return LIB
    BUILD.mkdir(parents=True, exist_ok=True)
    cc = nvcc()
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []

    def compile_one(src: Path) -> Path:
        obj = BUILD / (src.stem + ".o")
        cmd = [cc, *ARCH, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stderr}")
        if verbose or ptxas_verbose:
            sys.stderr.write(r.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, _sources()))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [cc, *ARCH, "-shared", "-Xcompiler", "-fPIC", *map(str, objs), "-o", str(tmp), "-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


TORCH_EXT_DIR = PKG / "torch_ext"
TORCH_EXT_SRC = TORCH_EXT_DIR / "cuda_uva.cpp"


def torch_ext_path() -> Path:
    return TORCH_EXT_DIR / ("cuda_uva" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))


def build_torch_ext(force: bool = False) -> Path:
    """Compiles the cuda_uva torch extension (g++, torch and CUDA headers) against
    libmserve_kv.so; returns its path.  Rebuilt only when its source, the header or the library
    is newer than it."""
    lib = build(force=False)
    out = torch_ext_path()
    deps = [TORCH_EXT_SRC, INCLUDE / "mserve_kv.h", lib, Path(__file__)]
    if not force and out.exists() and all(p.stat().st_mtime <= out.stat().st_mtime for p in deps):
        return out
    import torch
    tdir = Path(torch.__file__).resolve().parent
    cuda_home = Path(nvcc()).resolve().parent.parent
    cxx = shutil.which("g++") or shutil.which("c++")
    if not cxx:
        raise RuntimeError("a C++ compiler (g++) is required to build the cuda_uva extension")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    tmp = out.with_suffix(".tmp")
    cmd = [cxx, "-O3", "-std=c++17", "-fPIC", "-shared", str(TORCH_EXT_SRC), "-o", str(tmp),
           "-DTORCH_EXTENSION_NAME=cuda_uva", "-DTORCH_API_INCLUDE_EXTENSION_H", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           f"-I{tdir / 'include'}", f"-I{tdir / 'include' / 'torch' / 'csrc' / 'api' / 'include'}",
           f"-I{cuda_home / 'include'}", f"-I{sysconfig.get_paths()['include']}", f"-I{INCLUDE}",
           f"-L{tdir / 'lib'}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
           f"-L{cuda_home / 'lib64'}", "-lcudart", f"-L{PKG}", "-l:libmserve_kv.so",
           "-Wl,-rpath,$ORIGIN/..", f"-Wl,-rpath,{tdir / 'lib'}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"building the cuda_uva extension failed:\n{r.stderr[-4000:]}")
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    force = "--force" in sys.argv
    path = build(force=force, verbose="-v" in sys.argv, ptxas_verbose="--ptxas" in sys.argv)
    print(path)
    print(build_torch_ext(force=force))
