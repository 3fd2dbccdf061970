"""Gather rate of the reference's own UVA kernel next to mskv_uva_gather (baseline timing).

Runs qwen-eljrte/cuda_uva_kernel.cpp as built unmodified by oracle/build_ref.py and this
library's mskv_uva_gather on the same pinned cache and pinned index list, after checking that
every pointer the reference kernel dereferences is device-accessible at its host address.
Each figure is the median of 5 alternating rounds (reference, then this library) of 20 calls
timed with CUDA events, after warm-up; bytes = K + V rows gathered.

    python -m oracle.time_reference_kernel
"""
from __future__ import annotations

import ctypes as C
import json

import torch

from oracle import build_ref

SHAPES = {   # name: (B, H, T, D, S)
    "harness default (B1 H8 T8192 D128 S2048)": (1, 8, 8192, 128, 2048),
    "one 7B layer as stored by the reference ([1,4,32768,128], 4096 rows)": (1, 4, 32768, 128, 4096),
    "one 7B decode layer of the bench (8 seqs x 4 heads, 2176 rows each, shared list)": (8, 4, 16384, 128, 2176),
}


def _same_address_on_device(t: torch.Tensor) -> bool:
    from mserve_b200 import _lib
    p = C.c_void_p()
    rc = _lib.lib().mskv_device_view(C.c_void_p(t.data_ptr()), C.byref(p))
    return rc == _lib.MSKV_OK and p.value == t.data_ptr()


def _time(fn, reps=20, warmup=3) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    e1.synchronize()
    return e0.elapsed_time(e1) / reps


def main():
    ref = build_ref.load()
    if ref is None:
        print(json.dumps({"unavailable": "oracle/_ref/cuda_uva_ref.so is not built"}))
        return
    from mserve_b200 import cuda_uva
    g = torch.Generator().manual_seed(0)
    out = []
    for name, (B, H, T, D, S) in SHAPES.items():
        k = torch.randn(B, H, T, D, generator=g).to(torch.bfloat16).pin_memory()
        v = torch.randn(B, H, T, D, generator=g).to(torch.bfloat16).pin_memory()
        idx = torch.randperm(T, generator=g)[:S].sort().values.to(torch.int64).pin_memory()
        if not all(_same_address_on_device(t) for t in (k, v, idx)):
            out.append({"shape": name, "skipped": "pinned memory not device-accessible at its host address"})
            continue
        nbytes = 2 * B * H * S * D * k.element_size()
        rounds_ref, rounds_own = [], []
        for _ in range(5):
            rounds_ref.append(_time(lambda: ref.uva_gather(k, v, idx, B, H, T, D)))
            rounds_own.append(_time(lambda: cuda_uva.uva_gather(k, v, idx, B, H, T, D)))
        ms_ref = sorted(rounds_ref)[2]
        ms_own = sorted(rounds_own)[2]
        rk, rv = ref.uva_gather(k, v, idx, B, H, T, D)
        ok, ov = cuda_uva.uva_gather(k, v, idx, B, H, T, D)
        torch.cuda.synchronize()
        out.append({"shape": name, "bytes": nbytes, "reference_kernel_ms": ms_ref,
                    "reference_kernel_gbs": nbytes / ms_ref / 1e6, "mskv_uva_gather_ms": ms_own,
                    "mskv_uva_gather_gbs": nbytes / ms_own / 1e6, "speedup": ms_ref / ms_own,
                    "bit_exact": bool(torch.equal(rk.view(torch.int16), ok.view(torch.int16))
                                      and torch.equal(rv.view(torch.int16), ov.view(torch.int16)))})
    for o in out:
        print(json.dumps(o))


if __name__ == "__main__":
    main()
