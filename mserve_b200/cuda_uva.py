"""Drop-in for MServe's ``cuda_uva`` extension.

``uva_gather`` keeps the name, argument order, output layout and error behaviour of the
reference binding (qwen-eljrte/cuda_uva_kernel.cpp:48-113, qwen-eljrte/cuda_uva_kernel_v2.cpp:86-133)
and runs the sm_100a row gather of libmserve_kv (mskv_uva_gather).  A caller switches with

    import mserve_b200.cuda_uva as cuda_uva      # instead of: import cuda_uva

Differences that are deliberate (all supersets of the reference behaviour):
  * the kernel is enqueued on torch's current CUDA stream and never synchronises the device
    (v2 ends with cudaDeviceSynchronize, cuda_uva_kernel_v2.cpp:127; v1 used the legacy
    default stream, cuda_uva_kernel.cpp:86);
  * indices may also be a CUDA tensor (the reference requires CPU indices and reads them
    through a host pointer from the device, cuda_uva_kernel.cpp:36, 62, 91);
  * indices are bounds-checked: CPU indices before the launch (RuntimeError), CUDA indices
    on the device (the row is zero-filled and ``check_errors()`` raises);
  * fp8 (e4m3fn / e5m2) KV is accepted -- the copy is bitwise for any element size;
  * 64-bit offsets (the reference computes offsets in ``int``, cuda_uva_kernel.cpp:24-40).
"""
from __future__ import annotations

from typing import List, Optional

import ctypes as C
import torch

from . import ops
from ._lib import check, lib


def _check_input(t: torch.Tensor, name: str) -> None:
    # Error texts follow the reference's TORCH_CHECKs (cuda_uva_kernel.cpp:58-62).
    if t.is_cuda:
        return
    if not t.is_pinned():
        raise RuntimeError(f"{name} must be pinned memory for UVA")


def uva_gather(k_in: torch.Tensor, v_in: torch.Tensor, indices: torch.Tensor, batch_size: int, num_heads: int,
               seq_len: int, head_dim: int) -> List[torch.Tensor]:
    """k_out[b,h,s,:] = k_in[b,h,indices[s],:] (same for V) -> [k_out, v_out] on the current device.

    k_in, v_in: pinned CPU tensors (or CUDA tensors) holding [batch_size, num_heads, seq_len,
    head_dim] contiguously; indices: int64 [S] on the CPU (or CUDA).  Outputs are new CUDA
    tensors [B, H, S, D] of k_in's dtype.
    """
    _check_input(k_in, "k_in")
    _check_input(v_in, "v_in")
    if not k_in.is_cuda and not k_in.is_cpu:
        raise RuntimeError("k_in must be on CPU (pinned)")
    if indices.device.type not in ("cpu", "cuda"):
        raise RuntimeError("indices must be on CPU")
    if k_in.dtype != v_in.dtype:
        raise RuntimeError("k_in and v_in must have the same dtype")
    if k_in.dtype not in ops.GATHER_DTYPES:
        raise RuntimeError(f'"uva_gather" not implemented for \'{k_in.dtype}\'')
    B, H, T, D = int(batch_size), int(num_heads), int(seq_len), int(head_dim)
    need = B * H * T * D
    for name, t in (("k_in", k_in), ("v_in", v_in)):
        if not t.is_contiguous():
            raise RuntimeError(f"{name} must be contiguous")
        if t.numel() < need:
            raise RuntimeError(f"{name} has {t.numel()} elements, fewer than B*H*T*D = {need}")
    if indices.dim() != 1:
        raise RuntimeError("indices must be 1-D [num_selected]")
    S = indices.shape[0]
    dev = torch.device("cuda", torch.cuda.current_device())
    k_out = torch.empty(B, H, S, D, dtype=k_in.dtype, device=dev)
    v_out = torch.empty(B, H, S, D, dtype=k_in.dtype, device=dev)
    if S == 0 or B * H * D == 0:
        return [k_out, v_out]
    if indices.is_cuda:
        idx = indices.to(device=dev, dtype=torch.int64).contiguous()
    else:
        idx64 = indices.to(torch.int64)
        lo, hi = int(idx64.min()), int(idx64.max())
        if lo < 0 or hi >= T:
            raise RuntimeError(f"indices out of range [0, {T}): min {lo}, max {hi}")
        # Asynchronous H2D of the index list from page-locked memory (a pinned staging copy
        # for pageable input; torch keeps the pinned block until the copy has run), so the
        # call never waits for earlier work on the stream.
        src = idx64.contiguous()
        if not src.is_pinned():
            src = src.pin_memory()
        idx = src.to(dev, non_blocking=True)
    status = ops.status_word(dev)
    stream = torch.cuda.current_stream(dev)
    check(lib().mskv_uva_gather(C.c_void_p(k_in.data_ptr()), C.c_void_p(v_in.data_ptr()),
                                C.c_void_p(idx.data_ptr()), S, B, H, T, D, k_in.element_size(),
                                C.c_void_p(k_out.data_ptr()), C.c_void_p(v_out.data_ptr()),
                                C.c_void_p(status.data_ptr()), C.c_void_p(stream.cuda_stream)))
    # Keep the device copy of the indices alive until the gather has run.
    idx.record_stream(stream)
    return [k_out, v_out]


def check_errors(device: Optional[torch.device] = None) -> None:
    """Raises RuntimeError if a gather on `device` met an out-of-range index (synchronising)."""
    ops.check_status(device or torch.device("cuda", torch.cuda.current_device()), "uva_gather")
