"""Torch-facing wrappers of the libmserve_kv entry points.

PyTorch supplies device memory, the current stream and dtypes; every byte of KV data is
moved or reduced by the sm_100a kernels behind ``include/mserve_kv.h``.  Each wrapper
validates shapes and strides on the host (raising ``ValueError``/``RuntimeError`` before any
launch), fills the C descriptor and launches on ``torch.cuda.current_stream()``.
"""
from __future__ import annotations

import ctypes as C
import math
import weakref
from dataclasses import dataclass
from typing import Optional, Sequence, Tuple

import numpy as np
import torch

from . import _lib
from ._lib import AttnDesc, CopyDesc, FilterDesc, GatherDesc, Rows, ScoreDesc, TopkDesc, check, lib

_DTYPE_CODE = {
    torch.float32: _lib.DT_F32,
    torch.float16: _lib.DT_F16,
    torch.bfloat16: _lib.DT_BF16,
    torch.float64: _lib.DT_F64,
    torch.float8_e4m3fn: _lib.DT_FP8_E4M3,
    torch.float8_e5m2: _lib.DT_FP8_E5M2,
}
# Element types the reference extension dispatches (AT_DISPATCH_FLOATING_TYPES_AND2(Half,
# BFloat16): float, double, half, bfloat16) plus the two fp8 KV formats.
GATHER_DTYPES = (torch.float32, torch.float64, torch.float16, torch.bfloat16,
                 torch.float8_e4m3fn, torch.float8_e5m2)
COMPUTE_DTYPES = (torch.float32, torch.float16, torch.bfloat16)


def _stream_ptr(stream: Optional[torch.cuda.Stream] = None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else int(t.data_ptr())


# ---------------------------------------------------------------------------------------
# device status word
# ---------------------------------------------------------------------------------------
_status: dict = {}


def status_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 word the kernels OR status bits into (MSKV_STATUS_*)."""
    dev = torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    w = _status.get(idx)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=f"cuda:{idx}")
        _status[idx] = w
    return w


def take_status(device: torch.device) -> int:
    """Synchronises the current stream and returns the device status bits, clearing them."""
    w = status_word(device)
    v = int(w.item())
    if v:
        w.zero_()
    return v


def describe_status(v: int) -> str:
    reasons = []
    if v & _lib.STATUS_INDEX_OOB:
        reasons.append("token index out of range")
    if v & _lib.STATUS_BAD_PAGE:
        reasons.append("page-table entry not mapped")
    if v & _lib.STATUS_DST_OOB:
        reasons.append("destination token out of range")
    if v & _lib.STATUS_TIMEOUT:
        reasons.append("a wait for another GPU's flag timed out")
    return f"{', '.join(reasons)} (status 0x{v:x})"


def check_status(device: torch.device, what: str = "kernel") -> None:
    """Synchronises the current stream, raises RuntimeError if any status bit is set, clears it."""
    v = take_status(device)
    if v:
        raise RuntimeError(f"{what}: {describe_status(v)}; offending rows were skipped")


# ---------------------------------------------------------------------------------------
# pinned, mapped host memory
# ---------------------------------------------------------------------------------------
def _free_host(ptr: int) -> None:
    try:
        lib().mskv_host_free(C.c_void_p(ptr))
    except Exception:
        pass


def host_empty(shape: Sequence[int], dtype: torch.dtype) -> torch.Tensor:
    """CPU tensor in pinned, device-mapped, portable host memory (cudaHostAlloc).

    Every GPU of the process can read and write it in place.  The memory is released when
    the last tensor (or view) referencing it is garbage collected; callers must keep it
    alive until kernels using it have completed.
    """
    es = torch.empty((), dtype=dtype).element_size()
    n = int(np.prod(shape)) * es
    nbytes = max(n, 16)
    p = C.c_void_p()
    check(lib().mskv_host_alloc(C.byref(p), nbytes))
    buf = (C.c_uint8 * nbytes).from_address(p.value)
    arr = np.ctypeslib.as_array(buf)
    weakref.finalize(arr, _free_host, p.value)
    t = torch.from_numpy(arr)[:n].view(dtype)
    return t.view(*shape) if len(shape) else t.view(())


def device_view_ok(t: torch.Tensor) -> bool:
    """True when the tensor's memory can be dereferenced by the GPU (device or mapped pinned)."""
    if t.is_cuda:
        return True
    if t.numel() == 0:
        return True
    p = C.c_void_p()
    return lib().mskv_device_view(C.c_void_p(t.data_ptr()), C.byref(p)) == _lib.MSKV_OK


# ---------------------------------------------------------------------------------------
# row addressing
# ---------------------------------------------------------------------------------------
@dataclass
class RowsSpec:
    """Python mirror of mskv_rows plus the tensors that must stay alive with it."""
    rows: Rows
    keep: tuple
    row_bytes: int
    heads: int
    dtype: torch.dtype


def _norm(device) -> torch.device:
    d = torch.device(device)
    if d.type == "cuda" and d.index is None:
        d = torch.device("cuda", torch.cuda.current_device())
    return d


def _i32_or_none(t: Optional[torch.Tensor], name: str, device: torch.device) -> Optional[torch.Tensor]:
    if t is None:
        return None
    if t.dtype != torch.int32 or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous int32 tensor")
    if _norm(t.device) != _norm(device) and not (t.device.type == "cpu" and device_view_ok(t)):
        raise ValueError(f"{name} must live on {device} (or in mapped pinned memory)")
    return t


def strided_rows(k: torch.Tensor, v: Optional[torch.Tensor] = None, *, len_: Optional[torch.Tensor] = None,
                 len_scalar: Optional[int] = None, ring_start: Optional[torch.Tensor] = None,
                 ring_cap: int = 0, tok0: Optional[torch.Tensor] = None,
                 device: Optional[torch.device] = None) -> RowsSpec:
    """Rows of a [B, H, T, D] tensor (any strides, unit stride on D); T is the token axis."""
    if k.dim() != 4:
        raise ValueError(f"expected a [B, H, T, D] tensor, got shape {tuple(k.shape)}")
    if k.stride(3) != 1:
        raise ValueError("the head_dim axis must be contiguous")
    if v is not None and (v.shape != k.shape or v.stride() != k.stride() or v.dtype != k.dtype):
        raise ValueError("k and v must have the same shape, strides and dtype")
    es = k.element_size()
    dev = device or torch.device("cuda", torch.cuda.current_device())
    r = Rows()
    r.base_k = k.data_ptr() if k.numel() else None
    r.base_v = v.data_ptr() if (v is not None and v.numel()) else None
    r.stride_b, r.stride_h, r.stride_t = k.stride(0) * es, k.stride(1) * es, k.stride(2) * es
    r.len_scalar = k.shape[2] if len_scalar is None else int(len_scalar)
    r.len = _ptr(_i32_or_none(len_, "len", dev))
    r.ring_start = _ptr(_i32_or_none(ring_start, "ring_start", dev))
    r.ring_cap = int(ring_cap)
    r.tok0 = _ptr(_i32_or_none(tok0, "tok0", dev))
    return RowsSpec(r, (k, v, len_, ring_start, tok0), k.shape[3] * es, k.shape[1], k.dtype)


def paged_rows(k_pool: torch.Tensor, v_pool: Optional[torch.Tensor], page_table: torch.Tensor, *,
               len_: Optional[torch.Tensor] = None, len_scalar: Optional[int] = None,
               tok0: Optional[torch.Tensor] = None) -> RowsSpec:
    """Rows of a paged pool [P, H, page_size, D] addressed through page_table [B, max_pages]."""
    if k_pool.dim() != 4 or k_pool.stride(3) != 1:
        raise ValueError("pool must be [P, H, page_size, D] with a contiguous head_dim")
    if v_pool is not None and (v_pool.shape != k_pool.shape or v_pool.stride() != k_pool.stride()):
        raise ValueError("k and v pools must match")
    if page_table.dim() != 2 or page_table.dtype != torch.int32 or page_table.stride(1) != 1:
        raise ValueError("page_table must be int32 [B, max_pages] with unit inner stride")
    es = k_pool.element_size()
    dev = k_pool.device
    r = Rows()
    r.base_k = k_pool.data_ptr()
    r.base_v = v_pool.data_ptr() if v_pool is not None else None
    r.stride_page, r.stride_h, r.stride_t = k_pool.stride(0) * es, k_pool.stride(1) * es, k_pool.stride(2) * es
    r.page_table = page_table.data_ptr()
    r.pt_stride_b = page_table.stride(0)
    r.page_size = k_pool.shape[2]
    r.num_pages = k_pool.shape[0]
    r.len_scalar = page_table.shape[1] * k_pool.shape[2] if len_scalar is None else int(len_scalar)
    r.len = _ptr(_i32_or_none(len_, "len", dev))
    r.tok0 = _ptr(_i32_or_none(tok0, "tok0", dev))
    return RowsSpec(r, (k_pool, v_pool, page_table, len_, tok0), k_pool.shape[3] * es, k_pool.shape[1],
                    k_pool.dtype)


# ---------------------------------------------------------------------------------------
# gather / copy
# ---------------------------------------------------------------------------------------
def gather(src: RowsSpec, indices: torch.Tensor, out_k: torch.Tensor, out_v: Optional[torch.Tensor] = None,
           *, batch: int, counts: Optional[torch.Tensor] = None, status: bool = True,
           stream: Optional[torch.cuda.Stream] = None, max_ctas: int = 0) -> None:
    """out[b,h,s,:] = src[b,h,indices[...,s],:] for s < count(b,h) (mskv_gather).

    max_ctas: grid bound (0: the library's default, bounded for host memory).

    indices: int32/int64, shape [S] (shared by all segments), [B, S] (shared by the heads of
    a sequence) or [B, H, S] (one list per segment), contiguous, on the output's device.
    out_k/out_v: [B, H, S, D] device tensors with unit stride on D.
    """
    heads = src.heads
    if indices.dtype not in (torch.int32, torch.int64) or not indices.is_contiguous():
        raise ValueError("indices must be a contiguous int32 or int64 tensor")
    S = indices.shape[-1]
    if indices.dim() == 1:
        isb, ish = 0, 0
    elif indices.dim() == 2:
        if indices.shape[0] != batch:
            raise ValueError("indices [B, S] must have B == batch")
        isb, ish = S, 0
    elif indices.dim() == 3:
        if indices.shape[0] != batch or indices.shape[1] != heads:
            raise ValueError("indices [B, H, S] must match (batch, heads)")
        isb, ish = heads * S, S
    else:
        raise ValueError("indices must be 1-D, 2-D or 3-D")
    if out_k.shape != (batch, heads, S, src.row_bytes // out_k.element_size()) or out_k.stride(3) != 1:
        raise ValueError(f"out_k must be [B={batch}, H={heads}, S={S}, D] with contiguous D, got {tuple(out_k.shape)}")
    if out_k.element_size() * out_k.shape[3] != src.row_bytes:
        raise ValueError("output row size differs from the source row size")
    if src.rows.base_v and out_v is None:
        raise ValueError("source has V rows but out_v is None")
    if not out_k.is_cuda:
        raise ValueError("outputs must be CUDA tensors")
    dst = strided_rows(out_k, out_v, device=out_k.device)
    d = GatherDesc()
    d.src = src.rows
    d.dst = dst.rows
    d.indices = indices.data_ptr() if indices.numel() else None
    d.idx_stride_b, d.idx_stride_h = isb, ish
    if counts is not None:
        if counts.dtype != torch.int32 or not counts.is_contiguous() or counts.numel() not in (batch, batch * heads):
            raise ValueError("counts must be contiguous int32 [B] or [B, H]")
        d.counts = counts.data_ptr()
        d.cnt_stride_b, d.cnt_stride_h = (heads, 1) if counts.numel() == batch * heads else (1, 0)
    d.row_bytes = src.row_bytes
    d.status = status_word(out_k.device).data_ptr() if status else None
    d.index_bits = 64 if indices.dtype == torch.int64 else 32
    d.batch, d.heads, d.num_selected = batch, heads, S
    d.max_ctas = int(max_ctas)
    check(lib().mskv_gather(C.byref(d), _stream_ptr(stream)))


def copy_rows(src: RowsSpec, dst: RowsSpec, *, batch: int, num_tokens: int,
              counts: Optional[torch.Tensor] = None, device: Optional[torch.device] = None,
              status: bool = True, stream: Optional[torch.cuda.Stream] = None, max_ctas: int = 0) -> None:
    """Row i < count[b] of every (b,h): dst[b,h,dst.tok0[b]+i] = src[b,h,src.tok0[b]+i] (mskv_copy_rows).

    max_ctas: grid bound (0: the library's default, bounded for host memory)."""
    if src.row_bytes != dst.row_bytes or src.heads != dst.heads:
        raise ValueError("source and destination rows differ in size or head count")
    dev = device or torch.device("cuda", torch.cuda.current_device())
    d = CopyDesc()
    d.src, d.dst = src.rows, dst.rows
    if counts is not None:
        if counts.dtype != torch.int32 or counts.numel() != batch:
            raise ValueError("counts must be int32 [B]")
        d.counts = counts.data_ptr()
    d.row_bytes = src.row_bytes
    d.status = status_word(dev).data_ptr() if status else None
    d.batch, d.heads, d.num_tokens = batch, src.heads, num_tokens
    d.max_ctas = int(max_ctas)
    check(lib().mskv_copy_rows(C.byref(d), _stream_ptr(stream)))


# ---------------------------------------------------------------------------------------
# scoring / selection
# ---------------------------------------------------------------------------------------
def score(q: torch.Tensor, k: RowsSpec, *, batch: int, kv_heads: int, max_tokens: int,
          out: torch.Tensor, method: int = 0, stream: Optional[torch.cuda.Stream] = None,
          peers: Sequence[int] = ()) -> torch.Tensor:
    """fp32 importance of every token per (b, KV head) (mskv_score).

    q: [B, Hq, D] (or [B, Hq, 1, D]) in the K dtype; out: fp32 [B, Hkv, >= max_tokens].
    method 0: GQA-summed q·k; method 1: ||k||_2.  peers: device addresses of up to 7 other
    copies of `out` (same layout, mapped from other GPUs): every score is stored there too
    (mskv_score_fanout).
    """
    if q.dim() == 4:
        q = q[:, :, -1, :]
    if q.dim() != 3 or q.stride(2) != 1:
        raise ValueError("q must be [B, Hq, D] with contiguous D")
    Hq, D = q.shape[1], q.shape[2]
    if Hq % kv_heads:
        raise ValueError("q heads must be a multiple of kv heads")
    if q.dtype != k.dtype:
        raise ValueError(f"q dtype {q.dtype} differs from K dtype {k.dtype}")
    if k.dtype not in COMPUTE_DTYPES:
        raise TypeError(f"scoring supports float32/float16/bfloat16 keys, got {k.dtype}")
    if out.dtype != torch.float32 or out.dim() != 3 or out.stride(2) != 1 or out.shape[0] != batch \
            or out.shape[1] != kv_heads or out.shape[2] < max_tokens or out.stride(0) != kv_heads * out.stride(1):
        raise ValueError("out must be fp32 [B, Hkv, >= max_tokens] with rows at a common stride")
    d = ScoreDesc()
    d.k = k.rows
    d.q = q.data_ptr()
    es = q.element_size()
    d.q_stride_b, d.q_stride_h = q.stride(0) * es, q.stride(1) * es
    d.scores = out.data_ptr()
    d.scores_stride = out.stride(1)
    d.max_tokens = max_tokens
    d.status = status_word(out.device).data_ptr()
    d.dtype = _DTYPE_CODE[k.dtype]
    d.method = method
    d.batch, d.q_heads, d.kv_heads, d.head_dim = batch, Hq, kv_heads, D
    keep = (q, out, k)
    if peers:
        arr = (C.c_void_p * len(peers))(*[int(p) for p in peers])
        check(lib().mskv_score_fanout(C.byref(d), arr, len(peers), _stream_ptr(stream)))
    else:
        check(lib().mskv_score(C.byref(d), _stream_ptr(stream)))
    del keep
    return out


def blocked_layout(blocks: int, num_sel: int, rows_per_block: int, row_len: int) -> Tuple[int, int, int]:
    """(sel_stride, row_block, block_stride) of a contiguous [blocks, num_sel, rows_per_block,
    row_len] score tensor: row r of selection j starts at
    j*sel_stride + (r // row_block)*block_stride + (r % row_block)*row_len."""
    return rows_per_block * row_len, rows_per_block, num_sel * rows_per_block * row_len


def topk(scores: torch.Tensor, *, top_k, recent: int = 0, len_: Optional[torch.Tensor] = None,
         len_scalar: Optional[int] = None, rows_per_sel: int = 1, sel_per_batch: int = 1,
         scale: float = 1.0, out: Optional[torch.Tensor] = None, counts: Optional[torch.Tensor] = None,
         out_dtype: torch.dtype = torch.int32, stream: Optional[torch.cuda.Stream] = None,
         row_blocks: Optional[tuple] = None, k_bound: Optional[int] = None):
    """Sorted top-k ∪ recent-window indices per selection (mskv_topk).

    scores: fp32 [num_rows, >= T] with a common row stride (num_rows = num_sel*rows_per_sel).
    top_k: int, or int32 device tensor [B] (per sequence); k_bound, when given, bounds every
    top_k[b] (the caller knows it on the host: no device read, so the call can be captured).
    row_blocks: (blocks, num_sel, rows_per_block) for scores laid out as a contiguous
    [blocks, num_sel, rows_per_block, T] tensor (per-head score rows all-gathered from the
    ranks that hold the heads); selection j then sums its blocks*rows_per_block rows in
    block-major order, i.e. in global head order.
    Returns (idx [num_sel, K_max + recent], counts int32 [num_sel]).
    """
    if scores.dtype != torch.float32 or scores.stride(-1) != 1:
        raise ValueError("scores must be fp32 with a contiguous token axis")
    sel_stride = block_stride = row_block = 0
    if row_blocks is not None:
        nblk, nsel_b, rpb = (int(x) for x in row_blocks)
        if not scores.is_contiguous() or scores.numel() != nblk * nsel_b * rpb * scores.shape[-1]:
            raise ValueError("row_blocks needs a contiguous [blocks, num_sel, rows_per_block, T] tensor")
        rows = scores.reshape(-1, scores.shape[-1])
        if rows_per_sel != nblk * rpb:
            raise ValueError("rows_per_sel must equal blocks * rows_per_block")
        num_sel = nsel_b
        sel_stride, row_block, block_stride = blocked_layout(nblk, nsel_b, rpb, rows.shape[1])
    else:
        rows = scores.reshape(-1, scores.shape[-1]) if scores.is_contiguous() else scores
        if rows.dim() != 2:
            raise ValueError("scores must be 2-D or contiguous")
        if rows.shape[0] % rows_per_sel:
            raise ValueError("number of score rows must be a multiple of rows_per_sel")
        num_sel = rows.shape[0] // rows_per_sel
    T = rows.shape[1] if len_scalar is None else int(len_scalar)
    if T > rows.shape[1]:
        raise ValueError("len_scalar exceeds the score rows")
    dev = scores.device
    if isinstance(top_k, torch.Tensor):
        if top_k.dtype != torch.int32 or not top_k.is_contiguous():
            raise ValueError("per-sequence top_k must be contiguous int32")
        if k_bound is not None:
            k_max = int(k_bound)
        else:
            k_max = int(top_k.max().item()) if top_k.numel() else 0
        k_ptr, k_scalar = top_k.data_ptr(), 0
    else:
        k_max, k_ptr, k_scalar = int(top_k), None, int(top_k)
    width = max(0, min(k_max, T)) + max(0, int(recent))
    if out is None:
        out = torch.empty(num_sel, max(width, 1), dtype=out_dtype, device=dev)
    if counts is None:
        counts = torch.empty(num_sel, dtype=torch.int32, device=dev)
    if out.dim() != 2 or out.shape[0] != num_sel or out.shape[1] < width or out.stride(1) != 1:
        raise ValueError("out must be [num_sel, >= K + recent] with unit inner stride")
    d = TopkDesc()
    d.scores = rows.data_ptr()
    d.scores_stride = rows.stride(0)
    d.out_idx = out.data_ptr()
    d.out_stride = out.stride(0)
    d.counts = counts.data_ptr()
    d.len = _ptr(_i32_or_none(len_, "len", dev))
    d.top_k = k_ptr
    d.status = None
    d.scale = float(scale)
    d.len_scalar = T
    d.top_k_scalar = k_scalar
    d.recent = int(recent)
    d.num_sel, d.rows_per_sel, d.sel_per_batch = num_sel, rows_per_sel, sel_per_batch
    d.out_bits = 64 if out.dtype == torch.int64 else 32
    d.row_block, d.sel_stride, d.block_stride = row_block, sel_stride, block_stride
    check(lib().mskv_topk(C.byref(d), _stream_ptr(stream)))
    return out, counts


# ---------------------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------------------
_workspaces: dict = {}


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    key = (device.index, torch.cuda.current_stream(device).cuda_stream)
    w = _workspaces.get(key)
    if w is None or w.numel() < nbytes:
        w = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
        _workspaces[key] = w
    return w


def sparse_attention(q: torch.Tensor, k_sel: torch.Tensor, v_sel: torch.Tensor, *,
                     counts: Optional[torch.Tensor] = None, scale: Optional[float] = None,
                     out: Optional[torch.Tensor] = None, workspace: Optional[torch.Tensor] = None,
                     stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """softmax(scale·q·K_selᵀ)·V_sel per KV-head group (mskv_sparse_attention).

    q: [B, Hq, Q, D]; k_sel/v_sel: [B, Hk, S, D] with Hq % Hk == 0 and contiguous (S, D);
    counts: int32 [B, Hk] valid rows (None: all S).  Returns [B, Hq, Q, D] in q's dtype.
    """
    if q.dim() != 4 or k_sel.dim() != 4 or v_sel.shape != k_sel.shape:
        raise ValueError("q must be [B,Hq,Q,D] and k_sel/v_sel [B,Hk,S,D]")
    B, Hq, Q, D = q.shape
    Bk, Hk, S, Dk = k_sel.shape
    if Bk != B or Dk != D or Hq % Hk:
        raise ValueError(f"shape mismatch: q {tuple(q.shape)} vs k_sel {tuple(k_sel.shape)}")
    if q.dtype != k_sel.dtype or v_sel.dtype != k_sel.dtype or q.dtype not in COMPUTE_DTYPES:
        raise TypeError("q, k_sel, v_sel must share a float32/float16/bfloat16 dtype")
    es = q.element_size()
    for name, t in (("k_sel", k_sel), ("v_sel", v_sel)):
        if t.stride(3) != 1 or t.stride(2) != D or t.stride(0) != Hk * t.stride(1):
            raise ValueError(f"{name} must have contiguous [S, D] rows and uniform segment stride")
    if k_sel.stride() != v_sel.stride():
        raise ValueError("k_sel and v_sel must share strides")
    if q.stride(3) != 1:
        raise ValueError("q must have a contiguous head_dim")
    if out is None:
        out = torch.empty(B, Hq, Q, D, dtype=q.dtype, device=q.device)
    d = AttnDesc()
    d.q = q.data_ptr()
    d.q_stride_b, d.q_stride_h, d.q_stride_q = q.stride(0) * es, q.stride(1) * es, q.stride(2) * es
    d.k, d.v = k_sel.data_ptr(), v_sel.data_ptr()
    d.kv_stride_seg, d.kv_stride_s = k_sel.stride(1) * es, k_sel.stride(2) * es
    if counts is not None:
        if counts.dtype != torch.int32 or counts.numel() != B * Hk or not counts.is_contiguous():
            raise ValueError("counts must be contiguous int32 [B, Hk]")
        d.counts = counts.data_ptr()
    d.out = out.data_ptr()
    d.out_stride_b, d.out_stride_h, d.out_stride_q = out.stride(0) * es, out.stride(1) * es, out.stride(2) * es
    d.scale = float(scale if scale is not None else 1.0 / math.sqrt(D))
    d.status = status_word(q.device).data_ptr()
    d.dtype = _DTYPE_CODE[q.dtype]
    d.batch, d.q_heads, d.kv_heads, d.head_dim, d.q_len, d.num_selected = B, Hq, Hk, D, Q, S
    need = int(lib().mskv_attention_workspace_bytes(C.byref(d)))
    if need:
        ws = workspace if workspace is not None else _workspace(q.device, need)
        if ws.numel() * ws.element_size() < need:
            raise ValueError(f"workspace needs {need} bytes")
        d.workspace = ws.data_ptr()
        d.workspace_bytes = ws.numel() * ws.element_size()
    check(lib().mskv_sparse_attention(C.byref(d), _stream_ptr(stream)))
    return out


# ---------------------------------------------------------------------------------------
# prefill image-token filter
# ---------------------------------------------------------------------------------------
def image_filter(attn0: torch.Tensor, *, img_start: int, img_seq: int, text_start: int, text_seq: int,
                 global_thr: float, individual_thr: float, round_f16: bool = False,
                 stream: Optional[torch.cuda.Stream] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Kept image tokens of one attention map (mskv_image_filter).

    attn0: [H, Q, K] attention probabilities of one sequence (fp32/fp16/bf16, any strides);
    image tokens are the keys [img_start, +img_seq), text tokens the query rows
    [text_start, +text_seq).  round_f16 (fp32 input only) rounds every element to fp16 first and
    computes the stages in fp16, as the reference's use_fp16 does.  Returns (idx int64
    [img_seq] of which the first count entries are the kept image tokens in ascending order,
    count int32 [1]), both on attn0's device, without synchronising.
    """
    if attn0.dim() != 3 or not attn0.is_cuda:
        raise ValueError("attn0 must be a CUDA tensor [H, Q, K]")
    if attn0.dtype not in COMPUTE_DTYPES:
        raise TypeError(f"attention probabilities must be float32/float16/bfloat16, got {attn0.dtype}")
    if round_f16 and attn0.dtype != torch.float32:
        raise ValueError("round_f16 applies to float32 probabilities only")
    H, Q, K = attn0.shape
    if (img_start < 0 or img_seq < 0 or text_start < 0 or text_seq <= 0 or img_start + img_seq > K
            or text_start + text_seq > Q):
        raise ValueError(f"image keys [{img_start}, +{img_seq}) / text rows [{text_start}, +{text_seq}) "
                         f"do not fit a [{Q}, {K}] map")
    dev = attn0.device
    s = stream if stream is not None else torch.cuda.current_stream(dev)
    with torch.cuda.stream(s):          # outputs and workspace belong to the launching stream
        idx = torch.empty(max(img_seq, 1), dtype=torch.int64, device=dev)
        count = torch.empty(1, dtype=torch.int32, device=dev)
        ws = torch.empty(max(int(lib().mskv_image_filter_workspace_bytes(img_seq, text_seq)), 4), dtype=torch.uint8,
                         device=dev)
    d = FilterDesc()
    d.attn = attn0.data_ptr()
    d.stride_h, d.stride_q, d.stride_k = attn0.stride(0), attn0.stride(1), attn0.stride(2)
    d.out_idx, d.out_count = idx.data_ptr(), count.data_ptr()
    d.workspace, d.workspace_bytes = ws.data_ptr(), ws.numel()
    d.global_thr, d.individual_thr = float(global_thr), float(individual_thr)
    d.dtype = _DTYPE_CODE[attn0.dtype]
    d.heads, d.img_start, d.img_seq = H, int(img_start), int(img_seq)
    d.text_start, d.text_seq = int(text_start), int(text_seq)
    d.round_f16 = int(bool(round_f16))
    keep = (attn0, idx, count, ws)
    check(lib().mskv_image_filter(C.byref(d), _stream_ptr(s)))
    del keep
    return idx, count


# ---------------------------------------------------------------------------------------
# peer memory and flags (CUDA IPC; the score-row exchange between the GPUs of one node)
# ---------------------------------------------------------------------------------------
def ipc_alloc(nbytes: int) -> Tuple[int, bytes]:
    """Zeroed device memory that other processes can map: (address, IPC handle bytes)."""
    n = int(lib().mskv_ipc_handle_bytes())
    handle = C.create_string_buffer(n)
    ptr = C.c_void_p()
    check(lib().mskv_ipc_alloc(int(nbytes), C.byref(ptr), handle))
    return int(ptr.value), handle.raw


def ipc_open(handle: bytes) -> int:
    """Maps another process's mskv_ipc_alloc memory into this one; returns its address here."""
    buf = C.create_string_buffer(bytes(handle), len(handle))
    ptr = C.c_void_p()
    check(lib().mskv_ipc_open(buf, C.byref(ptr)))
    return int(ptr.value)


def ipc_close(ptr: int) -> None:
    check(lib().mskv_ipc_close(C.c_void_p(ptr)))


def ipc_free(ptr: int) -> None:
    check(lib().mskv_ipc_free(C.c_void_p(ptr)))


def flag_signal(flag_arrays: Sequence[int], index: int, value: int, stream: Optional[torch.cuda.Stream] = None):
    """Stores `value` at element `index` of every int64 flag array, after the stream's earlier work."""
    arr = (C.c_void_p * len(flag_arrays))(*[int(p) for p in flag_arrays])
    check(lib().mskv_flag_signal(arr, len(flag_arrays), int(index), int(value), _stream_ptr(stream)))


def flag_wait(flags: int, count: int, value: int, *, at_least: bool = False, timeout_s: float = 1.0,
              device: Optional[torch.device] = None, stream: Optional[torch.cuda.Stream] = None):
    """Makes the stream wait until the `count` int64 flags at `flags` equal (or reach) `value`;
    after timeout_s the wait gives up and sets the timeout status bit (check_status raises)."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    check(lib().mskv_flag_wait(C.c_void_p(int(flags)), int(count), int(value), int(bool(at_least)),
                               int(timeout_s * 1e9), C.c_void_p(status_word(dev).data_ptr()), _stream_ptr(stream)))


class _DeviceArray:
    """A device address range seen as a tensor (the CUDA array interface, no copy)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"data": (int(ptr), False), "shape": tuple(shape), "typestr": typestr,
                                         "version": 3, "strides": None}


def device_tensor(ptr: int, shape, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    """A tensor over device memory this library allocated (the caller keeps it alive)."""
    typestr = {torch.float32: "<f4", torch.int64: "<i8", torch.int32: "<i4"}[dtype]
    return torch.as_tensor(_DeviceArray(ptr, shape, typestr), device=device)