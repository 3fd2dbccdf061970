"""Builds the reference's own UVA gather extension -- test infrastructure, not product code.

qwen-eljrte/cuda_uva_kernel.cpp is CUDA source under a .cpp name: the shipped setup script
(qwen-eljrte/setup_cuda_uva.py:16-30) hands it to g++, which cannot compile a kernel launch.
This recipe compiles it where it lies, unmodified, as CUDA (nvcc -x cu) for sm_100a against the
installed torch, into oracle/_ref/cuda_uva_ref.so (Python module ``cuda_uva_ref``, the only
name that changes: TORCH_EXTENSION_NAME).  Nothing is copied out of the reference tree; the
build output goes to oracle/_ref/ only, which travels to the GPU machine with the repository.

Users: tests/test_reference_kernel_gpu.py (bit-exact cross-check of mskv_uva_gather against
the reference kernel) and oracle/time_reference_kernel.py (the reference kernel's gather rate).

    python -m oracle.build_ref [--force] [--reference <MServe checkout>]

The reference checkout comes from --reference or the MSERVE_REFERENCE environment variable;
without either, an existing build is kept and nothing is compiled.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path
from typing import Optional

REF_FILE = "qwen-eljrte/cuda_uva_kernel.cpp"
OUT_DIR = Path(__file__).resolve().parent / "_ref"
OUT = OUT_DIR / "cuda_uva_ref.so"
MODULE = "cuda_uva_ref"


def reference_source(reference: Optional[str] = None) -> Optional[Path]:
    """The reference kernel source under `reference` (default: $MSERVE_REFERENCE), if present."""
    root = reference or os.environ.get("MSERVE_REFERENCE")
    if not root:
        return None
    src = Path(root) / REF_FILE
    return src if src.exists() else None


def build(force: bool = False, reference: Optional[str] = None) -> Optional[Path]:
    """Returns the built module path, or None when neither the source nor a build exists."""
    REF_SOURCE = reference_source(reference)
    if REF_SOURCE is None:
        return OUT if OUT.exists() else None
    if OUT.exists() and not force and OUT.stat().st_mtime >= REF_SOURCE.stat().st_mtime:
        return OUT
    import torch
    import torch.utils.cpp_extension as ce
    nvcc = shutil.which("nvcc") or os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
    includes = [os.path.join(os.path.dirname(torch.__file__), "include"),
                os.path.join(os.path.dirname(torch.__file__), "include", "torch", "csrc", "api", "include"),
                os.path.join(os.path.dirname(nvcc), "..", "include"),
                sysconfig.get_paths()["include"]]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    OUT_DIR.mkdir(exist_ok=True)
    cmd = [nvcc, "-x", "cu", str(REF_SOURCE), "-o", str(OUT), "-shared", "-Xcompiler", "-fPIC", "-O3",
           "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
           f"-DTORCH_EXTENSION_NAME={MODULE}", "-DTORCH_API_INCLUDE_EXTENSION_H", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           *[f"-I{p}" for p in includes], f"-L{torch_lib}",
           "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python", "-lcudart",
           "-Xlinker", f"-rpath,{torch_lib}"]
    subprocess.run(cmd, check=True)
    del ce
    return OUT


def load():
    """Imports the built reference module (oracle/_ref on sys.path); None when not built."""
    if not OUT.exists():
        return None
    if str(OUT_DIR) not in sys.path:
        sys.path.insert(0, str(OUT_DIR))
    import importlib
    return importlib.import_module(MODULE)


if __name__ == "__main__":
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--reference", default=None, help="root of an MServe checkout (default: $MSERVE_REFERENCE)")
    a = ap.parse_args()
    print(build(force=a.force, reference=a.reference))
