"""The B200 KV offload engine: host KV store + HBM key pages + the decode-step hot path.

Storage (per layer):
  * host store: pinned, device-mapped K and V, [B, Hkv, C, D] (the reference layout of
    CPUKVCache's host tensors, qwen-eljrte/Qwen_Transformer/kv_cache.py:14, 763, but with
    KV heads instead of repeat_kv'd query heads and a fixed capacity C).  Logical token t of
    sequence b lives at slot (ring_start[b] + t) mod C.  This is the gather source.
  * HBM key pages: K in 16-token pages, pool [P, Hkv, 16, D], one int32 page table
    [B, max_pages] shared by all layers.  This is what the scoring kernel reads, so a decode
    step never moves the full layer over PCIe (the reference copies the whole layer to the
    GPU every step, kv_cache.py:241-294 driven from qwen-eljrte/llm.py:131-197).

Append (prefill chunk or decode token), per layer: the new K rows are scattered into their
HBM pages (mskv_copy_rows, paged destination) and the new K and V rows are written through
to the host store (mskv_copy_rows, ring destination, zero-copy PCIe stores).

Decode step, per layer (``decode_layer``): GQA-summed fp32 scores from the HBM pages
(mskv_score) -> top-k of [0, L-R) plus the recent window [L-R, L) per (sequence, KV head)
(mskv_topk) -> gather of the selected K/V rows from the host store into HBM
(mskv_gather) -> attention over them (mskv_sparse_attention).  No host synchronisation.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence

import numpy as np
import torch

from . import ops


@dataclass
class DecodeBuffers:
    """Per-engine reusable device buffers of one decode layer."""
    scores: torch.Tensor      # fp32 [B, Hkv, T_cap]
    idx: torch.Tensor         # int32 [B*Hkv, S]
    counts: torch.Tensor      # int32 [B*Hkv]
    k_sel: torch.Tensor       # [B, Hkv, S, D]
    v_sel: torch.Tensor
    out: torch.Tensor         # [B, Hq, 1, D]


class OffloadKV:
    """Host-resident KV with HBM key pages for a fixed batch of sequences.

    num_layers, batch, q_heads, kv_heads, head_dim: model/batch geometry.
    capacity: tokens per sequence in the host store (and in the page table).
    top_k, recent: the selection per (sequence, KV head): top_k tokens of [0, L - recent)
    plus the last `recent` tokens.
    """

    def __init__(self, num_layers: int, batch: int, q_heads: int, kv_heads: int, head_dim: int, capacity: int, *,
                 top_k: int, recent: int = 0, dtype: torch.dtype = torch.bfloat16, page_size: int = 16,
                 device: Optional[torch.device] = None, host_alloc=None):
        if q_heads % kv_heads:
            raise ValueError("q_heads must be a multiple of kv_heads")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.L, self.B, self.Hq, self.Hkv, self.D = num_layers, batch, q_heads, kv_heads, head_dim
        self.C, self.page_size, self.dtype = capacity, page_size, dtype
        self.top_k, self.recent = int(top_k), int(recent)
        self.S = self.top_k + self.recent
        alloc = host_alloc or ops.host_empty
        self.host_k: List[torch.Tensor] = [alloc((batch, kv_heads, capacity, head_dim), dtype) for _ in range(num_layers)]
        self.host_v: List[torch.Tensor] = [alloc((batch, kv_heads, capacity, head_dim), dtype) for _ in range(num_layers)]
        self.max_pages = (capacity + page_size - 1) // page_size
        self.num_pages = batch * self.max_pages
        self.pool_k: List[torch.Tensor] = [
            torch.empty(self.num_pages, kv_heads, page_size, head_dim, dtype=dtype, device=self.device)
            for _ in range(num_layers)]
        # Page ids are handed out from a free list as sequences grow.
        self._free = list(range(self.num_pages - 1, -1, -1))
        self.page_table_h = np.full((batch, self.max_pages), -1, dtype=np.int32)
        self.page_table = torch.full((batch, self.max_pages), -1, dtype=torch.int32, device=self.device)
        self.len_h = np.zeros(batch, dtype=np.int64)
        self.lens = torch.zeros(batch, dtype=torch.int32, device=self.device)
        self.ring_start = torch.zeros(batch, dtype=torch.int32, device=self.device)
        self._pending = None
        self._bufs: Optional[DecodeBuffers] = None

    # ------------------------------------------------------------------ append
    def reserve(self, n_new: Sequence[int]) -> None:
        """Starts an append of n_new[b] tokens per sequence: maps the pages they need.

        Every layer must then be given its rows with ``append_layer`` before ``commit``.
        """
        n_new = np.asarray(n_new, dtype=np.int64).reshape(self.B)
        if self._pending is not None:
            raise RuntimeError("reserve() called twice without commit()")
        new_len = self.len_h + n_new
        if (new_len > self.C).any():
            raise ValueError(f"append exceeds the store capacity of {self.C} tokens per sequence")
        for b in range(self.B):
            first = int(self.len_h[b]) // self.page_size
            last = (int(new_len[b]) + self.page_size - 1) // self.page_size
            for p in range(first, last):
                if self.page_table_h[b, p] < 0:
                    if not self._free:
                        raise RuntimeError("HBM key-page pool exhausted")
                    self.page_table_h[b, p] = self._free.pop()
        self.page_table.copy_(torch.from_numpy(self.page_table_h), non_blocking=False)
        self._pending = (n_new, torch.from_numpy(self.len_h.astype(np.int32)).to(self.device),
                         torch.from_numpy(n_new.astype(np.int32)).to(self.device))

    def append_layer(self, layer: int, k_new: torch.Tensor, v_new: torch.Tensor) -> None:
        """Rows [B, Hkv, n, D] (n >= max n_new) of one layer: HBM key pages + host write-through."""
        if self._pending is None:
            raise RuntimeError("append_layer() outside reserve()/commit()")
        n_new, tok0, counts = self._pending
        n = k_new.shape[2]
        if k_new.shape[:2] != (self.B, self.Hkv) or k_new.shape[3] != self.D or n < int(n_new.max(initial=0)):
            raise ValueError(f"k_new must be [B={self.B}, Hkv={self.Hkv}, >= n_new, D={self.D}]")
        if k_new.dtype != self.dtype or v_new.dtype != self.dtype or v_new.shape != k_new.shape:
            raise ValueError("k_new/v_new dtype or shape mismatch")
        src = ops.strided_rows(k_new, v_new, device=self.device)
        src_k_only = ops.strided_rows(k_new, None, device=self.device)
        pages = ops.paged_rows(self.pool_k[layer], None, self.page_table, len_scalar=self.C)
        pages.rows.tok0 = tok0.data_ptr()
        host = ops.strided_rows(self.host_k[layer], self.host_v[layer], len_scalar=self.C,
                                ring_start=self.ring_start, ring_cap=self.C, tok0=tok0, device=self.device)
        ops.copy_rows(src_k_only, pages, batch=self.B, num_tokens=n, counts=counts, device=self.device)
        ops.copy_rows(src, host, batch=self.B, num_tokens=n, counts=counts, device=self.device)
        del src, src_k_only, pages, host

    def commit(self) -> None:
        """Ends the append started by ``reserve``: the new tokens become visible."""
        if self._pending is None:
            raise RuntimeError("commit() without reserve()")
        n_new, tok0, counts = self._pending
        self.len_h = self.len_h + n_new
        self.lens.copy_(torch.from_numpy(self.len_h.astype(np.int32)), non_blocking=False)
        # tok0/counts were read by kernels on the current stream; keep them alive until then.
        cur = torch.cuda.current_stream(self.device)
        tok0.record_stream(cur)
        counts.record_stream(cur)
        self._pending = None

    # ------------------------------------------------------------------ decode
    def buffers(self) -> DecodeBuffers:
        if self._bufs is None:
            dev, B, Hkv, S, D = self.device, self.B, self.Hkv, self.S, self.D
            self._bufs = DecodeBuffers(
                scores=torch.empty(B, Hkv, self.C, dtype=torch.float32, device=dev),
                idx=torch.empty(B * Hkv, max(S, 1), dtype=torch.int32, device=dev),
                counts=torch.empty(B * Hkv, dtype=torch.int32, device=dev),
                k_sel=torch.empty(B, Hkv, max(S, 1), D, dtype=self.dtype, device=dev),
                v_sel=torch.empty(B, Hkv, max(S, 1), D, dtype=self.dtype, device=dev),
                out=torch.empty(B, self.Hq, 1, D, dtype=self.dtype, device=dev))
        return self._bufs

    def select(self, layer: int, q: torch.Tensor, bufs: Optional[DecodeBuffers] = None):
        """Scores + top-k ∪ window for one layer; returns (idx [B*Hkv, S], counts [B*Hkv])."""
        bufs = bufs or self.buffers()
        T = int(self.len_h.max(initial=0))
        keys = ops.paged_rows(self.pool_k[layer], None, self.page_table, len_=self.lens)
        ops.score(q, keys, batch=self.B, kv_heads=self.Hkv, max_tokens=T, out=bufs.scores, method=0)
        ops.topk(bufs.scores.view(self.B * self.Hkv, self.C), top_k=self.top_k, recent=self.recent,
                 len_=self.lens, len_scalar=T, rows_per_sel=1, sel_per_batch=self.Hkv,
                 out=bufs.idx, counts=bufs.counts)
        return bufs.idx, bufs.counts

    def gather(self, layer: int, idx: torch.Tensor, counts: torch.Tensor, bufs: Optional[DecodeBuffers] = None):
        """Selected K/V rows from the host store into HBM [B, Hkv, S, D]."""
        bufs = bufs or self.buffers()
        src = ops.strided_rows(self.host_k[layer], self.host_v[layer], len_=self.lens,
                               ring_start=self.ring_start, ring_cap=self.C, device=self.device)
        ops.gather(src, idx.view(self.B, self.Hkv, -1), bufs.k_sel, bufs.v_sel, batch=self.B,
                   counts=counts.view(self.B, self.Hkv))
        return bufs.k_sel, bufs.v_sel

    def attend(self, q: torch.Tensor, counts: torch.Tensor, bufs: Optional[DecodeBuffers] = None) -> torch.Tensor:
        bufs = bufs or self.buffers()
        q4 = q.unsqueeze(2) if q.dim() == 3 else q
        return ops.sparse_attention(q4, bufs.k_sel, bufs.v_sel, counts=counts.view(self.B, self.Hkv), out=bufs.out)

    def decode_layer(self, layer: int, q: torch.Tensor) -> torch.Tensor:
        """One layer of the decode hot path; q [B, Hq, D] -> attention output [B, Hq, 1, D]."""
        bufs = self.buffers()
        idx, counts = self.select(layer, q, bufs)
        self.gather(layer, idx, counts, bufs)
        return self.attend(q, counts, bufs)

    # ------------------------------------------------------------------ views for tests / baselines
    def host_logical(self, layer: int, b: int):
        """Logical-order host K/V of sequence b (CPU tensors [Hkv, len, D])."""
        n = int(self.len_h[b])
        st = int(self.ring_start[b].item())
        idx = (st + torch.arange(n)) % self.C
        return self.host_k[layer][b][:, idx], self.host_v[layer][b][:, idx]

    def kernels_per_decode_layer(self) -> int:
        return 5  # score, topk, gather, attention partial + combine
