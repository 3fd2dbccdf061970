"""gcc recipe for oracle/liboracle_kv.so (test infrastructure: the C restatement used as the
timed CPU baseline).  ``python -m oracle.build_oracle`` or via ``__graft_entry__.build()``.

Compiled for x86-64-v3 (AVX2/FMA) so the library built here also runs on the GPU box's host.
"""
from __future__ import annotations

import ctypes as C
import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "oracle_kv.c"
LIB = HERE / "liboracle_kv.so"
FLAGS = ["-O3", "-march=x86-64-v3", "-fopenmp", "-fPIC", "-shared", "-std=c11", "-ffp-contract=off"]


def build(force: bool = False) -> Path:
    if not force and LIB.exists() and LIB.stat().st_mtime >= max(SRC.stat().st_mtime, Path(__file__).stat().st_mtime):
        return LIB
    cc = shutil.which("gcc") or "cc"
    tmp = LIB.with_suffix(".so.tmp")
    r = subprocess.run([cc, *FLAGS, str(SRC), "-o", str(tmp), "-lm"], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"gcc failed:\n{r.stderr}")
    tmp.replace(LIB)
    return LIB


_lib = None


def load() -> C.CDLL:
    global _lib
    if _lib is None:
        build()
        h = C.CDLL(str(LIB))
        vp, i64, i32 = C.c_void_p, C.c_int64, C.c_int
        h.okv_max_threads.restype = i32
        h.okv_gather.argtypes = [vp, vp, i64, i64, i64, i32, i32, vp, i32, i64, i64, i32, vp, vp, vp, i64, i32]
        h.okv_score_bf16.argtypes = [vp, vp, i64, i64, i64, i32, i32, i32, i32, i32, vp, i64, i32]
        h.okv_topk.argtypes = [vp, i64, i32, i32, vp, i32, i32, i32, vp, i64, vp, i32]
        h.okv_attention_bf16.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32, i32, C.c_float, vp, i32]
        _lib = h
    return _lib


if __name__ == "__main__":
    print(build(force=True))
