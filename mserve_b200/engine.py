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
to the host store (mskv_copy_rows, ring destination, zero-copy PCIe stores).  A decode loop
appends its own token inside the step: begin_step() grows the lengths without a host
synchronisation, decode_step(..., k_new, v_new) writes each layer's token before that
layer's selection, and a step captured with a length bound replays as the cache grows.

Decode step, per layer (``decode_layer``): GQA-summed fp32 scores from the HBM pages
(mskv_score) -> top-k of [0, L-R) plus the recent window [L-R, L) per (sequence, KV head)
(mskv_topk) -> gather of the selected K/V rows from the host store into HBM
(mskv_gather) -> attention over them (mskv_sparse_attention).  No host synchronisation.
``decode_step`` pipelines these over sequence chunks and four streams and prefetches each
layer's recent-window rows; ``capture_decode_step`` captures the whole step as a CUDA graph.
"""
from __future__ import annotations

import contextlib
import math
from dataclasses import dataclass
from typing import List, Optional, Sequence

import numpy as np
import torch

from . import ops, topology


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
    plus the last `recent` tokens.  top_k_ratio instead of top_k: ceil(top_k_ratio * L_b)
    tokens for sequence b, following each sequence's length.
    For KV heads sharded over GPUs, each rank builds its engine with its own heads (kv_heads =
    its share, q_heads = the matching query heads); per-head selection needs no exchange.
    """

    def __init__(self, num_layers: int, batch: int, q_heads: int, kv_heads: int, head_dim: int, capacity: int, *,
                 top_k: int = 0, recent: int = 0, top_k_ratio: Optional[float] = None,
                 dtype: torch.dtype = torch.bfloat16, page_size: int = 16,
                 device: Optional[torch.device] = None, host_alloc=None, numa_local: bool = True):
        if q_heads % kv_heads:
            raise ValueError("q_heads must be a multiple of kv_heads")
        if top_k_ratio is not None and not 0.0 < top_k_ratio <= 1.0:
            raise ValueError("top_k_ratio must lie in (0, 1]")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.L, self.B, self.Hq, self.Hkv, self.D = num_layers, batch, q_heads, kv_heads, head_dim
        self.C, self.page_size, self.dtype = capacity, page_size, dtype
        self.top_k, self.recent = int(top_k), int(recent)
        self.top_k_ratio = top_k_ratio
        # per-sequence k (host copy and device copy), refreshed by commit()
        self.topk_h = np.zeros(batch, dtype=np.int64)
        self.topk_dev = torch.zeros(batch, dtype=torch.int32, device=self.device)
        k_cap = math.ceil(top_k_ratio * capacity) if top_k_ratio is not None else self.top_k
        self.S = k_cap + self.recent
        alloc = host_alloc or ops.host_empty
        # The host store goes on the NUMA node of this GPU's PCIe link (numa_local).
        placement = topology.local_placement(self.device) if numa_local else contextlib.nullcontext(set())
        with placement as cpus:
            self.host_cpus = cpus
            self.host_k: List[torch.Tensor] = [alloc((batch, kv_heads, capacity, head_dim), dtype)
                                               for _ in range(num_layers)]
            self.host_v: List[torch.Tensor] = [alloc((batch, kv_heads, capacity, head_dim), dtype)
                                               for _ in range(num_layers)]
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
        # Per-sequence split of a selection (refreshed by commit): the top-k part holds k'_b =
        # min(k_b, n_b) rows, n_b = max(L_b - recent, 0), and the recent window the w_b = L_b - n_b
        # tokens [n_b, L_b) at output rows [k'_b, k'_b + w_b).  [n_b, k'_b, w_b] per sequence.
        self.split = torch.zeros(3, batch, dtype=torch.int32, device=self.device)
        self._pending = None
        self._bufs: Optional[DecodeBuffers] = None
        self._sel2 = None
        # Decode-token appends (begin_step + decode_step with k_new/v_new): the new token's
        # position per sequence, a count of one per sequence, and pinned staging for the
        # host-computed lengths, splits, per-sequence k and page table, guarded by an event.
        self.tok_new = torch.zeros(batch, dtype=torch.int32, device=self.device)
        self.ones_b = torch.ones(batch, dtype=torch.int32, device=self.device)
        self._stage = torch.empty(6 * batch, dtype=torch.int32).pin_memory()
        self._pt_stage = torch.empty(batch, self.max_pages, dtype=torch.int32).pin_memory()
        self._stage_ev: Optional[torch.cuda.Event] = None
        # CTAs of every move that reads host memory (the gathers and the window copies); 0: the
        # library's default bound
        self.host_link_ctas = 0

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
        split = self._refresh_split()
        if self.top_k_ratio is not None:
            self.topk_dev.copy_(torch.from_numpy(self.topk_h.astype(np.int32)), non_blocking=False)
        self.split.copy_(torch.from_numpy(split), non_blocking=False)
        # tok0/counts were read by kernels on the current stream; keep them alive until then.
        cur = torch.cuda.current_stream(self.device)
        tok0.record_stream(cur)
        counts.record_stream(cur)
        self._pending = None

    def _refresh_split(self) -> np.ndarray:
        """Per-sequence k (top_k_ratio) and the [n_b, k'_b, w_b] split for the host lengths."""
        if self.top_k_ratio is not None:
            self.topk_h = np.array([math.ceil(self.top_k_ratio * int(n)) for n in self.len_h], dtype=np.int64)
        n = np.maximum(self.len_h - self.recent, 0)
        k = self.topk_h if self.top_k_ratio is not None else np.full(self.B, self.top_k, dtype=np.int64)
        return np.stack([n, np.minimum(k, n), self.len_h - n]).astype(np.int32)

    def begin_step(self) -> None:
        """Room for one new token per sequence, for a decode_step given k_new/v_new.

        Maps a page for every sequence whose token starts one, and sets the device-side
        lengths, selection splits, per-sequence k and the new token's position (tok_new, the
        length before the step) -- through pinned staging copies on the current stream, with
        no host synchronisation (the host waits only for the previous step's staging copies).
        The step then scores and selects over the grown cache, the new token included, as the
        reference's decode scores over cat(past, new) (qwen-eljrte/Qwen_Transformer/
        kv_cache.py:631-643); decode_step writes the token itself.
        """
        if self._pending is not None:
            raise RuntimeError("begin_step() inside reserve()/commit()")
        if (self.len_h + 1 > self.C).any():
            raise ValueError(f"a decode token exceeds the store capacity of {self.C} tokens per sequence")
        mapped = False
        for b in range(self.B):
            p = int(self.len_h[b]) // self.page_size
            if self.page_table_h[b, p] < 0:
                if not self._free:
                    raise RuntimeError("HBM key-page pool exhausted")
                self.page_table_h[b, p] = self._free.pop()
                mapped = True
        if self._stage_ev is not None:
            self._stage_ev.synchronize()        # the staging buffers' last copies are done
        B = self.B
        old = self.len_h
        self.len_h = self.len_h + 1
        split = self._refresh_split()
        st = self._stage.numpy()
        st[0:B] = self.len_h
        st[B:2 * B] = old
        st[2 * B:5 * B] = split.reshape(-1)
        st[5 * B:6 * B] = self.topk_h
        if mapped:
            self._pt_stage.numpy()[:] = self.page_table_h
            self.page_table.copy_(self._pt_stage, non_blocking=True)
        self.lens.copy_(self._stage[0:B], non_blocking=True)
        self.tok_new.copy_(self._stage[B:2 * B], non_blocking=True)
        self.split.copy_(self._stage[2 * B:5 * B].view(3, B), non_blocking=True)
        if self.top_k_ratio is not None:
            self.topk_dev.copy_(self._stage[5 * B:6 * B], non_blocking=True)
        self._stage_ev = torch.cuda.Event()
        self._stage_ev.record(torch.cuda.current_stream(self.device))

    def _append_token(self, layer: int, k_tok: torch.Tensor, v_tok: torch.Tensor) -> None:
        """The step's token [B, Hkv, D] of one layer: K into its HBM page, K and V written
        through to the host store, at position tok_new of every sequence (begin_step)."""
        k4, v4 = k_tok.unsqueeze(2), v_tok.unsqueeze(2)
        src = ops.strided_rows(k4, v4, device=self.device)
        src_k_only = ops.strided_rows(k4, None, device=self.device)
        pages = ops.paged_rows(self.pool_k[layer], None, self.page_table, len_scalar=self.C, tok0=self.tok_new)
        host = ops.strided_rows(self.host_k[layer], self.host_v[layer], len_scalar=self.C,
                                ring_start=self.ring_start, ring_cap=self.C, tok0=self.tok_new, device=self.device)
        ops.copy_rows(src_k_only, pages, batch=self.B, num_tokens=1, counts=self.ones_b, device=self.device)
        ops.copy_rows(src, host, batch=self.B, num_tokens=1, counts=self.ones_b, device=self.device)

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
        top_k, k_bound = self._top_k(0, self.B)
        ops.topk(bufs.scores.view(self.B * self.Hkv, self.C), top_k=top_k, recent=self.recent,
                 len_=self.lens, len_scalar=T, rows_per_sel=1, sel_per_batch=self.Hkv,
                 out=bufs.idx, counts=bufs.counts, k_bound=k_bound)
        return bufs.idx, bufs.counts

    def _top_k(self, b0: int, b1: int, t_bound: Optional[int] = None):
        """(top_k argument, host bound) of sequences [b0, b1) for ops.topk; with t_bound the
        bound covers every length up to t_bound (a step replayed while the cache grows)."""
        if self.top_k_ratio is None:
            return self.top_k, None
        if t_bound is not None:
            return self.topk_dev[b0:b1], math.ceil(self.top_k_ratio * int(t_bound))
        return self.topk_dev[b0:b1], int(self.topk_h[b0:b1].max(initial=0))

    def gather(self, layer: int, idx: torch.Tensor, counts: torch.Tensor, bufs: Optional[DecodeBuffers] = None):
        """Selected K/V rows from the host store into HBM [B, Hkv, S, D]."""
        bufs = bufs or self.buffers()
        src = ops.strided_rows(self.host_k[layer], self.host_v[layer], len_=self.lens,
                               ring_start=self.ring_start, ring_cap=self.C, device=self.device)
        ops.gather(src, idx.view(self.B, self.Hkv, -1), bufs.k_sel, bufs.v_sel, batch=self.B,
                   counts=counts.view(self.B, self.Hkv), max_ctas=self.host_link_ctas)
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

    # ------------------------------------------------------------------ pipelined decode step
    def _host_rows(self, layer: int, b0: int, b1: int, tok0: Optional[torch.Tensor] = None) -> ops.RowsSpec:
        return ops.strided_rows(self.host_k[layer][b0:b1], self.host_v[layer][b0:b1], len_=self.lens[b0:b1],
                                ring_start=self.ring_start[b0:b1], ring_cap=self.C, tok0=tok0,
                                device=self.device)

    def _sel_rows(self, parity: int, bufs: DecodeBuffers):
        """Selected-row buffers (k_sel, v_sel) of set `parity`: layers alternate between two
        sets in the pipelined step, so one layer's window rows can land while the previous
        layer's attention still reads its own rows."""
        if parity == 0:
            return bufs.k_sel, bufs.v_sel
        if self._sel2 is None:
            self._sel2 = (torch.empty_like(bufs.k_sel), torch.empty_like(bufs.v_sel))
        return self._sel2

    def _window_rows(self, layer: int, k_sel: torch.Tensor, v_sel: torch.Tensor) -> None:
        """The recent-window rows of every sequence (tokens [n_b, L_b) -> rows [k'_b, k'_b + w_b)):
        they are selected whatever the scores, so they can move before the query exists."""
        if self.recent <= 0:
            return
        n0, kp, w = self.split[0], self.split[1], self.split[2]
        dst = ops.strided_rows(k_sel, v_sel, tok0=kp, device=self.device)
        ops.copy_rows(self._host_rows(layer, 0, self.B, tok0=n0), dst, batch=self.B, num_tokens=self.recent,
                      counts=w, device=self.device, max_ctas=self.host_link_ctas)

    def _chunk_ops(self, layer: int, q: torch.Tensor, b0: int, b1: int, bufs: DecodeBuffers, T: int,
                   sel_rows=None, window_done: bool = False):
        """Kernels of one layer for sequences [b0, b1): (select, gather, attend) closures.

        window_done: the window rows are already in sel_rows (see _window_rows), so the gather
        moves only the top-k part of each selection."""
        Hkv, C = self.Hkv, self.C
        nb = b1 - b0
        lens = self.lens[b0:b1]
        scores = bufs.scores[b0:b1]
        idx = bufs.idx[b0 * Hkv:b1 * Hkv]
        counts = bufs.counts[b0 * Hkv:b1 * Hkv]
        k_all, v_all = sel_rows if sel_rows is not None else (bufs.k_sel, bufs.v_sel)
        k_sel, v_sel = k_all[b0:b1], v_all[b0:b1]
        gcounts = self.split[1][b0:b1] if window_done and self.recent > 0 else counts

        def select():
            keys = ops.paged_rows(self.pool_k[layer], None, self.page_table[b0:b1], len_=lens)
            ops.score(q[b0:b1], keys, batch=nb, kv_heads=Hkv, max_tokens=T, out=scores, method=0)
            top_k, k_bound = self._top_k(b0, b1, T)
            ops.topk(scores.view(nb * Hkv, C), top_k=top_k, recent=self.recent, len_=lens, len_scalar=T,
                     rows_per_sel=1, sel_per_batch=Hkv, out=idx, counts=counts, k_bound=k_bound)

        def gather():
            ops.gather(self._host_rows(layer, b0, b1), idx.view(nb, Hkv, -1), k_sel, v_sel, batch=nb,
                       counts=gcounts.view(nb, -1), max_ctas=self.host_link_ctas)

        def attend(out):
            ops.sparse_attention(q[b0:b1].unsqueeze(2), k_sel, v_sel, counts=counts.view(nb, Hkv), out=out[b0:b1])

        return select, gather, attend

    def decode_step(self, q_all: torch.Tensor, out_all: torch.Tensor, chunks: int = 4, streams=None, *,
                    k_new: Optional[torch.Tensor] = None, v_new: Optional[torch.Tensor] = None,
                    t_bound: Optional[int] = None) -> None:
        """All layers of one decode step, pipelined over sequence chunks.

        q_all: [L, B, Hq, D]; out_all: [L, B, Hq, 1, D]; chunks: a number of equal chunks or
        the list of chunk sizes (sequences).  Within a layer, chunk c's scores and
        selection run on the caller's stream, its gather on one of two gather streams
        (alternating, so consecutive gathers overlap at their boundaries) and its attention on
        a fourth, so the selection of chunk c+1 and the attention of chunk c-1 execute while
        chunk c's rows cross PCIe.  Layer l+1 starts only after layer l's attention (the model
        dependency).  The side streams fork from and join back into the caller's stream, so
        the call can be captured in a CUDA graph.  The recent-window rows of layer l+1 (known
        before its query) are copied while layer l finishes, into the second of two alternating
        selected-row buffer sets.  Outputs are bit-identical to decode_layer.

        k_new, v_new: [L, B, Hkv, D], the step's own token of every layer, after begin_step():
        layer l's token is written (its HBM page and the host store) on the caller's stream
        before layer l's selection, and before its window rows are copied.  t_bound: the
        length bound that the kernels are launched for (default: the current longest
        sequence); a step captured with t_bound >= the current lengths stays valid while
        begin_step grows them up to t_bound.
        """
        bufs = self.buffers()
        T = int(self.len_h.max(initial=0))
        if t_bound is not None:
            if not T <= int(t_bound) <= self.C:
                raise ValueError(f"t_bound {t_bound} must lie in [{T}, {self.C}]")
            T = int(t_bound)
        append = k_new is not None or v_new is not None
        if append:
            want = (self.L, self.B, self.Hkv, self.D)
            if (k_new is None or v_new is None or tuple(k_new.shape) != want or tuple(v_new.shape) != want
                    or k_new.dtype != self.dtype or v_new.dtype != self.dtype):
                raise ValueError(f"k_new and v_new must both be {self.dtype} {list(want)}")
        cur = torch.cuda.current_stream(self.device)
        s_g0, s_g1, s_att = streams or self._side_streams()
        gat_streams = (s_g0, s_g1)
        bounds = self.chunk_bounds(chunks)
        n_chunks = len(bounds) - 1
        s_win = gat_streams[(n_chunks - 1) % 2]     # the stream of each layer's last gather
        sel_rows = [self._sel_rows(0, bufs), self._sel_rows(1, bufs)]
        if append:
            self._append_token(0, k_new[0], v_new[0])
        start = torch.cuda.Event()
        start.record(cur)
        for st in (s_g0, s_g1, s_att):
            st.wait_event(start)
        win_ev = torch.cuda.Event()
        with torch.cuda.stream(s_win):
            self._window_rows(0, *sel_rows[0])
            win_ev.record(s_win)
        for layer in range(self.L):
            sel_ev, gat_ev = [], []
            rows = sel_rows[layer % 2]
            parts = [self._chunk_ops(layer, q_all[layer], int(bounds[c]), int(bounds[c + 1]), bufs, T,
                                     sel_rows=rows, window_done=True)
                     for c in range(n_chunks)]
            for select, _, _ in parts:
                select()
                e = torch.cuda.Event()
                e.record(cur)
                sel_ev.append(e)
            # Chunk c's gather runs on gather stream c % 2, so the tail of one chunk's gather
            # overlaps the start of the next (the link stays busy across kernel boundaries).
            for c, ((_, gather, _), e) in enumerate(zip(parts, sel_ev)):
                st = gat_streams[c % 2]
                with torch.cuda.stream(st):
                    st.wait_event(e)
                    gather()
                    g = torch.cuda.Event()
                    g.record(st)
                    gat_ev.append(g)
            this_win = win_ev
            if layer + 1 < self.L:
                # The next layer's token goes in after this layer's selections (so before the
                # next layer's, on this stream) and before the next layer's window rows move.
                if append:
                    self._append_token(layer + 1, k_new[layer + 1], v_new[layer + 1])
                    app_ev = torch.cuda.Event()
                    app_ev.record(cur)
                # The next layer's window rows cross the link while this layer's last attention
                # and the next layer's first selection run.  Their buffer set was last read by
                # the attention of layer - 1, which finished before this layer's selections.
                win_ev = torch.cuda.Event()
                with torch.cuda.stream(s_win):
                    if append:
                        s_win.wait_event(app_ev)
                    self._window_rows(layer + 1, *sel_rows[(layer + 1) % 2])
                    win_ev.record(s_win)
            with torch.cuda.stream(s_att):
                s_att.wait_event(this_win)      # this layer's window rows are in place
                for (_, _, attend), g in zip(parts, gat_ev):
                    s_att.wait_event(g)
                    attend(out_all[layer])
                done = torch.cuda.Event()
                done.record(s_att)
            cur.wait_event(done)                # the next layer's query needs this layer's output
        for st in (s_g0, s_g1):
            end = torch.cuda.Event()
            end.record(st)
            cur.wait_event(end)

    def chunk_bounds(self, chunks) -> np.ndarray:
        """Sequence boundaries of the chunks: explicit chunk sizes, or a number of chunks.

        For a number n the first chunk holds one sequence -- its selection is the only one on
        the critical path of a layer, so the link starts as early as possible -- and the other
        B - 1 sequences are split as evenly as possible into n - 1 chunks."""
        if isinstance(chunks, (int, np.integer)):
            n = max(1, min(int(chunks), self.B))
            if n == 1:
                return np.array([0, self.B])
            rest = np.linspace(1, self.B, n).astype(int)      # n - 1 near-equal parts of [1, B)
            return np.concatenate([[0], rest]).astype(int)
        sizes = [int(c) for c in chunks]
        if not sizes or min(sizes) <= 0 or sum(sizes) != self.B:
            raise ValueError(f"chunk sizes {sizes} must be positive and sum to the batch {self.B}")
        return np.concatenate([[0], np.cumsum(sizes)]).astype(int)

    def _side_streams(self):
        """(gather stream 0, gather stream 1, attention stream)."""
        if getattr(self, "_streams", None) is None:
            self._streams = tuple(torch.cuda.Stream(self.device) for _ in range(3))
        return self._streams

    def capture_decode_step(self, q_all: torch.Tensor, out_all: torch.Tensor, chunks: int = 4, *,
                            k_new: Optional[torch.Tensor] = None, v_new: Optional[torch.Tensor] = None,
                            t_bound: Optional[int] = None):
        """CUDA graph of ``decode_step`` on fixed q/out (and k_new/v_new) buffers; returns the
        graph (``.replay()``).

        Replaying the graph launches every kernel of the step at once.  The buffers and the
        engine must stay alive while the graph is in use, and the lengths must stay within
        t_bound (default: the current longest sequence, i.e. the cache must not grow).  With
        k_new/v_new, each replay follows a begin_step() and writes that step's token; the
        capture itself runs the current step once (its warm-up), and replaying a step again
        rewrites the same token and recomputes the same outputs.
        """
        side = self._side_streams()
        kw = dict(k_new=k_new, v_new=v_new, t_bound=t_bound)
        self.decode_step(q_all, out_all, chunks, side, **kw)      # warm-up: allocates workspaces
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, capture_error_mode="relaxed"):
            self.decode_step(q_all, out_all, chunks, side, **kw)
        return g

    # ------------------------------------------------------------------ views for tests / baselines
    def host_logical(self, layer: int, b: int):
        """Logical-order host K/V of sequence b (CPU tensors [Hkv, len, D])."""
        n = int(self.len_h[b])
        st = int(self.ring_start[b].item())
        idx = (st + torch.arange(n)) % self.C
        return self.host_k[layer][b][:, idx], self.host_v[layer][b][:, idx]

    def kernels_per_decode_layer(self) -> int:
        return 5  # score, topk, gather, attention partial + combine
