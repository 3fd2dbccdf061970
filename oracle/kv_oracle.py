"""numpy restatement of MServe's KV selection-and-offload path (the oracle).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).  Every function cites the reference
file:line it restates (paths within the MServe project, prefix qwen-eljrte/).  Arrays are
numpy; bfloat16 data travels as uint16 bit patterns (``bf16_to_f32`` / ``f32_to_bf16``).

Parity contract with the CUDA path
  * gathers, appends and write-backs: bit-exact (byte copies);
  * scores: fp32 accumulation on the GPU vs. fp64 here, compared within 1e-3 relative;
  * selection: the kernel's rule restated exactly (``select_topk_window``) -- given the same
    fp32 scores the index sets are identical, ties resolved toward the lower token index;
  * attention: fp32 on the GPU vs. fp64 here, compared within 2e-2 relative in bf16.
"""
from __future__ import annotations

from typing import Optional, Sequence, Tuple, Union

import numpy as np

# ---------------------------------------------------------------------------------------
# bfloat16 helpers
# ---------------------------------------------------------------------------------------


def bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    """bfloat16 bit patterns (uint16) -> float32 (exact)."""
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(f: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns, round to nearest even (NaN kept quiet)."""
    u = np.asarray(f, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(f, dtype=np.float32))
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FC0
    return r


# ---------------------------------------------------------------------------------------
# (a1/a3) gather
# ---------------------------------------------------------------------------------------


def index_select_gather(k: np.ndarray, v: np.ndarray, indices: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """out[b,h,s,:] = in[b,h,indices[s],:] for K and V.

    Restates torch.index_select(k_cpu, dim=2, index=token_indices)
    (qwen-eljrte/Qwen_Transformer/kv_cache.py:597-599; qwen-eljrte/benchmark_kv_transfer.py:136-137)
    and the UVA kernel body (qwen-eljrte/cuda_uva_kernel.cpp:29-44): one index list shared by
    every (b, h), output order = index order, duplicates copied as given.
    """
    idx = np.asarray(indices, dtype=np.int64)
    T = k.shape[2]
    if idx.size and (idx.min() < -T or idx.max() >= T):
        raise IndexError("index out of range in index_select")
    return np.ascontiguousarray(k[:, :, idx, :]), np.ascontiguousarray(v[:, :, idx, :])


def gather_segments(src_k: np.ndarray, src_v: Optional[np.ndarray], indices: np.ndarray, *,
                    num_selected: Optional[int] = None, counts: Optional[np.ndarray] = None,
                    lens: Optional[np.ndarray] = None, ring_start: Optional[np.ndarray] = None,
                    ring_cap: int = 0):
    """Per-(b, KV head) gather from a (possibly ring-addressed) store [B, H, C, D].

    Generalises the reference gather (qwen-eljrte/cuda_uva_kernel.cpp:36-44) to one index
    list per segment ([S], [B,S] or [B,H,S]), a per-sequence valid length and a ring store in
    which logical token t of sequence b lives at physical slot (ring_start[b] + t) % ring_cap
    -- the in-place form of the reference's cat + keep-last-max_len host cache
    (qwen-eljrte/Qwen_Transformer/kv_cache.py:739-748).  Rows with an invalid index are
    zero-filled and reported.  Returns (k_out, v_out, valid_mask [B,H,S], oob_flag).
    """
    B, H, C, D = src_k.shape
    idx = np.asarray(indices, dtype=np.int64)
    S = idx.shape[-1] if num_selected is None else num_selected
    if idx.ndim == 1:
        idx = np.broadcast_to(idx, (B, H, idx.shape[0]))
    elif idx.ndim == 2:
        idx = np.broadcast_to(idx[:, None, :], (B, H, idx.shape[1]))
    L = np.full(B, C if lens is None else 0, dtype=np.int64) if lens is None else np.asarray(lens, dtype=np.int64)
    out_k = np.zeros((B, H, S) + src_k.shape[3:], dtype=src_k.dtype)
    out_v = None if src_v is None else np.zeros_like(out_k)
    mask = np.zeros((B, H, S), dtype=bool)
    oob = False
    for b in range(B):
        for h in range(H):
            n = S if counts is None else int(np.asarray(counts).reshape(B, -1)[b, h if np.asarray(counts).size == B * H else 0])
            n = min(n, S)
            for s in range(n):
                t = int(idx[b, h, s])
                mask[b, h, s] = True
                if t < 0 or t >= L[b]:
                    oob = True
                    continue
                p = t if ring_start is None else (int(ring_start[b]) + t) % ring_cap
                out_k[b, h, s] = src_k[b, h, p]
                if src_v is not None:
                    out_v[b, h, s] = src_v[b, h, p]
    return out_k, out_v, mask, oob


# ---------------------------------------------------------------------------------------
# (b) importance scores and selection
# ---------------------------------------------------------------------------------------


def repeat_kv(x: np.ndarray, n_rep: int) -> np.ndarray:
    """[B, Hkv, T, D] -> [B, Hkv*n_rep, T, D], head h -> h // n_rep.

    Restates repeat_kv (qwen-eljrte/Qwen_Transformer/attention.py:1701-1710)."""
    if n_rep == 1:
        return x
    return np.repeat(x, n_rep, axis=1)


def gqa_scores(q: np.ndarray, k: np.ndarray, *, lens: Optional[np.ndarray] = None, method: str = "attention_score",
               accum=np.float64) -> np.ndarray:
    """Per-(b, KV head) importance of every token.

    attention_score: s[b,hk,t] = sum_{g<G} q[b, hk*G+g, :] . k[b,hk,t,:]  -- the reference's
    per-head products q_last·Kᵀ (qwen-eljrte/Qwen_Transformer/attention.py:556-562) summed
    over the query heads that share KV head hk after repeat_kv (attention.py:1943-1944).
    norm: s[b,hk,t] = ||k[b,hk,t,:]||_2 (attention.py:574).
    q: [B, Hq, D] (or [B, Hq, Q, D]: the last query row is used, attention.py:556);
    k: [B, Hkv, T, D].  Tokens t >= lens[b] are set to NaN.  Returns [B, Hkv, T] in accum.
    """
    if q.ndim == 4:
        q = q[:, :, -1, :]
    B, Hq, D = q.shape
    _, Hkv, T, _ = k.shape
    G = Hq // Hkv
    kf = k.astype(accum)
    if method == "attention_score":
        qs = q.astype(accum).reshape(B, Hkv, G, D).sum(axis=2)
        s = np.einsum("bhd,bhtd->bht", qs, kf)
    elif method == "norm":
        s = np.sqrt((kf * kf).sum(axis=-1))
    else:
        raise ValueError(f"Unknown importance method: {method}")
    if lens is not None:
        for b in range(B):
            s[b, :, int(lens[b]):] = np.nan
    return s


def order_key(x: np.ndarray) -> np.ndarray:
    """Order-preserving map float32 -> uint32 (sign flip); every NaN maps to the top key."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32)
    k = np.where(u & np.uint32(0x80000000), ~u, u | np.uint32(0x80000000)).astype(np.uint32)
    return np.where((u & np.uint32(0x7FFFFFFF)) > np.uint32(0x7F800000), np.uint32(0xFFFFFFFF), k).astype(np.uint32)


def select_topk_window(rows: np.ndarray, *, top_k: Union[int, Sequence[int]], recent: int = 0,
                       lens: Optional[Sequence[int]] = None, len_scalar: Optional[int] = None,
                       rows_per_sel: int = 1, sel_per_batch: int = 1, scale: float = 1.0):
    """Top-k of the candidates [0, L - recent) plus the recent window [L - recent, L).

    The selection rule of mskv_topk, restated exactly:
      key(t) = float32(scale) * (rows[j*R] + rows[j*R+1] + ... + rows[j*R+R-1]) in fp32,
      summed in row order -- with R = number of heads and scale = 1/Hq this is the
      reference's scores.mean(dim=1) (qwen-eljrte/Qwen_Transformer/attention.py:565);
      k = min(top_k, n), n = max(L - recent, 0); ranking by key, ties toward the lower
      token index, NaN highest -- the reference's torch.topk(scores, k, sorted=False)
      (attention.py:567-572) plus a recent window the reference does not have.
    Returns (list of int64 arrays sorted ascending, counts).
    """
    rows = np.asarray(rows, dtype=np.float32)
    num_sel = rows.shape[0] // rows_per_sel
    T = rows.shape[1] if len_scalar is None else int(len_scalar)
    out, counts = [], []
    for j in range(num_sel):
        b = j // sel_per_batch
        L = T if lens is None else int(lens[b])
        n = max(L - recent, 0)
        K = top_k if np.isscalar(top_k) else top_k[b]
        K = max(0, min(int(K), n))
        key = rows[j * rows_per_sel, :n].astype(np.float32)
        for r in range(1, rows_per_sel):
            key = (key + rows[j * rows_per_sel + r, :n]).astype(np.float32)
        key = (key * np.float32(scale)).astype(np.float32)
        ok = order_key(key).astype(np.int64)
        order = np.lexsort((np.arange(n), -ok))
        sel = np.sort(order[:K]).astype(np.int64)
        sel = np.concatenate([sel, np.arange(n, L, dtype=np.int64)])
        out.append(sel)
        counts.append(len(sel))
    return out, np.asarray(counts, dtype=np.int32)


def compute_token_importance(query: np.ndarray, key: np.ndarray, method: str = "attention_score",
                             top_k_ratio: float = 0.3, min_tokens: int = 128, accum=np.float64) -> np.ndarray:
    """Restates compute_token_importance (qwen-eljrte/Qwen_Transformer/attention.py:532-588).

    query [B, H, Q, D]; key [B, Hk, T, D] with Hk dividing H (the reference passes repeat_kv'd
    keys, Hk == H).  scores = mean over the H query heads of q_last·kᵀ (or of ||k||), then
    k = min(max(min_tokens, int(T*top_k_ratio)), T) indices with the largest score.
    Returns int64 indices sorted ascending, shape [k] for B == 1 (the reference's
    .squeeze(0)) or [B, k].  Tie order among equal scores is unspecified in the reference
    (torch.topk, sorted=False); here the lower index wins.
    """
    B, H, Q, D = query.shape
    T = key.shape[2]
    Hk = key.shape[1]
    if method == "attention_score":
        per = gqa_scores(query[:, :, -1, :], key, accum=accum)    # [B, Hk, T]
        scores = per.sum(axis=1) / H
    elif method == "norm":
        per = gqa_scores(query, key, method="norm", accum=accum)
        scores = per.sum(axis=1) * (H // Hk) / H
    else:
        raise ValueError(f"Unknown importance method: {method}")
    k = max(min_tokens, int(T * top_k_ratio))
    k = min(k, T)
    out = np.empty((B, k), dtype=np.int64)
    for b in range(B):
        order = np.lexsort((np.arange(T), -scores[b]))
        out[b] = np.sort(order[:k])
    return out[0] if B == 1 else out


# ---------------------------------------------------------------------------------------
# attention over the selection
# ---------------------------------------------------------------------------------------


def sparse_sdpa_attention(q: np.ndarray, k_sel: np.ndarray, v_sel: np.ndarray, *,
                          counts: Optional[np.ndarray] = None, scale: Optional[float] = None,
                          accum=np.float64) -> np.ndarray:
    """softmax(scale * q·K_selᵀ)·V_sel, no mask.

    Restates sparse_sdpa_attention (qwen-eljrte/Qwen_Transformer/attention.py:619-636):
    attn_scores = matmul(q, k_sparseᵀ)/sqrt(D); softmax over the selected tokens; matmul with
    v_sparse.  k_sel/v_sel may hold Hk = Hq/G heads (query head hq uses KV head hq // G; the
    reference passes repeat_kv'd [B, Hq, S, D]).  counts [B, Hk] limits the rows per head.
    q [B, Hq, Q, D] -> [B, Hq, Q, D] in accum.
    """
    B, Hq, Q, D = q.shape
    Hk, S = k_sel.shape[1], k_sel.shape[2]
    G = Hq // Hk
    sc = 1.0 / np.sqrt(D) if scale is None else scale
    out = np.zeros((B, Hq, Q, D), dtype=accum)
    for b in range(B):
        for hq in range(Hq):
            hk = hq // G
            n = S if counts is None else int(np.asarray(counts).reshape(B, Hk)[b, hk])
            if n == 0:
                continue
            K = k_sel[b, hk, :n].astype(accum)
            V = v_sel[b, hk, :n].astype(accum)
            s = (q[b, hq].astype(accum) @ K.T) * sc
            s = s - s.max(axis=-1, keepdims=True)
            p = np.exp(s)
            p /= p.sum(axis=-1, keepdims=True)
            out[b, hq] = p @ V
    return out


# ---------------------------------------------------------------------------------------
# (c) append / write-back
# ---------------------------------------------------------------------------------------


def full_kv(past: Optional[Tuple[np.ndarray, np.ndarray]], new_k: np.ndarray, new_v: np.ndarray
            ) -> Tuple[np.ndarray, np.ndarray]:
    """CPUKVCache.get_full_kv (qwen-eljrte/Qwen_Transformer/kv_cache.py:631-643): the past K/V
    [B, H, T, D] followed by the new rows [B, H, n, D] along the token axis; no past: the new
    rows themselves."""
    if past is None:
        return new_k, new_v
    return (np.concatenate([past[0], new_k], axis=2), np.concatenate([past[1], new_v], axis=2))


def cat_truncate(old_k: Optional[np.ndarray], old_v: Optional[np.ndarray], new_k: np.ndarray, new_v: np.ndarray,
                 max_len: int) -> Tuple[np.ndarray, np.ndarray]:
    """Host-cache append: cat along tokens, keep the last max_len.

    Restates CPUKVCache.append_new (qwen-eljrte/Qwen_Transformer/kv_cache.py:733-748) and
    CPUKVCacheOptimized._append_cpu (kv_cache_optimized.py:126-139)."""
    if old_k is None:
        tk, tv = new_k, new_v
    else:
        tk = np.concatenate([old_k, new_k], axis=2)
        tv = np.concatenate([old_v, new_v], axis=2)
    if tk.shape[2] > max_len:
        tk = tk[:, :, -max_len:]
        tv = tv[:, :, -max_len:]
    return np.ascontiguousarray(tk), np.ascontiguousarray(tv)


class RingStore:
    """Ring-addressed host store: the in-place equivalent of cat_truncate.

    Logical token t of sequence b sits at physical slot (start[b] + t) % cap; appending n
    tokens writes them after the current end and, past capacity, advances start so the last
    cap tokens remain -- the same logical contents as kv_cache.py:739-748 without re-copying
    the old tokens.  Used to check the GPU write-back kernel bit-for-bit.
    """

    def __init__(self, B: int, H: int, cap: int, row_shape: Tuple[int, ...], dtype):
        self.k = np.zeros((B, H, cap) + row_shape, dtype=dtype)
        self.v = np.zeros_like(self.k)
        self.start = np.zeros(B, dtype=np.int64)
        self.len = np.zeros(B, dtype=np.int64)
        self.cap = cap

    def plan(self, n: int):
        """(dst logical token of the first kept new row, first kept new row, rows kept) per b,
        and the new (start, len) -- the host-side bookkeeping of one append of n rows."""
        plans = []
        for b in range(self.k.shape[0]):
            keep = min(n, self.cap)
            first_new = n - keep
            L = int(self.len[b])
            total = L + keep
            drop = max(0, total - self.cap)
            new_start = (int(self.start[b]) + drop) % self.cap
            new_len = total - drop
            dst_tok0 = L - drop     # logical position (after the shift) of the first kept row
            plans.append((dst_tok0, first_new, keep, new_start, new_len))
        return plans

    def append(self, new_k: np.ndarray, new_v: np.ndarray) -> None:
        n = new_k.shape[2]
        for b, (dst_tok0, first_new, keep, new_start, new_len) in enumerate(self.plan(n)):
            self.start[b], self.len[b] = new_start, new_len
            for i in range(keep):
                p = (new_start + dst_tok0 + i) % self.cap
                self.k[b, :, p] = new_k[b, :, first_new + i]
                self.v[b, :, p] = new_v[b, :, first_new + i]

    def logical(self, b: int):
        idx = (int(self.start[b]) + np.arange(int(self.len[b]))) % self.cap
        return self.k[b][:, idx], self.v[b][:, idx]


def paged_append(pool_k: np.ndarray, pool_v: np.ndarray, page_table: np.ndarray, seq_len: Sequence[int],
                 new_k: np.ndarray, new_v: np.ndarray, counts: Optional[Sequence[int]] = None) -> None:
    """Scatter new rows into 16-token (page_size) pages: token t = seq_len[b] + i of sequence b
    goes to pool[page_table[b, t // ps], :, t % ps, :].  In place.  (No reference counterpart:
    the reference re-copies the whole host cache per append, kv_cache.py:739-740.)"""
    ps = pool_k.shape[2]
    B, H, n = new_k.shape[:3]
    for b in range(B):
        c = n if counts is None else int(counts[b])
        for i in range(c):
            t = int(seq_len[b]) + i
            p = int(page_table[b, t // ps])
            pool_k[p, :, t % ps] = new_k[b, :, i]
            pool_v[p, :, t % ps] = new_v[b, :, i]


def page_writeback(pool_k: np.ndarray, pool_v: np.ndarray, page_table: np.ndarray, host_k: np.ndarray,
                   host_v: np.ndarray, tok_start: Sequence[int], counts: Sequence[int],
                   ring_start: Optional[Sequence[int]] = None, ring_cap: int = 0) -> None:
    """Write tokens [tok_start[b], tok_start[b] + counts[b]) of every sequence from the HBM
    pages to the host store (logical token t -> physical slot, ring-aware).  In place."""
    ps = pool_k.shape[2]
    for b in range(host_k.shape[0]):
        for i in range(int(counts[b])):
            t = int(tok_start[b]) + i
            p = int(page_table[b, t // ps])
            slot = t if ring_start is None else (int(ring_start[b]) + t) % ring_cap
            host_k[b, :, slot] = pool_k[p, :, t % ps]
            host_v[b, :, slot] = pool_v[p, :, t % ps]


def _stage(x, stage: str) -> np.ndarray:
    """Rounds float32 values to the stage dtype ('f32', 'f16' or 'bf16', nearest even)."""
    x = np.asarray(x, dtype=np.float32)
    if stage == "f16":
        return x.astype(np.float16).astype(np.float32)
    if stage == "bf16":
        u = x.view(np.uint32).astype(np.uint64)
        r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
        return r.astype(np.uint32).view(np.float32)
    if stage != "f32":
        raise ValueError(f"unknown stage dtype {stage}")
    return x


def image_filter_block(block: np.ndarray, global_thr: float, individual_thr: float, stage: str = "f32"):
    """The decision part of dual_attention_filter (qwen-eljrte/Qwen_Transformer/
    dual_attention_filter.py:47-70) on the text x image block [H, text, img] itself: rounded to
    the stage dtype (its .half() when use_fp16, line 47); head_mean = mean over heads (line 50);
    attn_sum = column sums over the text rows (line 54); text_max = column maxima (line 57); an
    image token is dropped when attn_sum < attn_sum.sum() * global_thr and text_max <
    individual_thr (line 62).  As torch tensors of the block's dtype, every stage result is
    rounded to `stage` ('f32', 'f16' or 'bf16'), the sums accumulating in float32.  The
    summation order is fixed: heads in order; text rows in blocks of 32, each summed in order
    and the block sums added in order; the total over tiles of 32 columns the same way.
    Returns (kept image-token indices ascending, attn_sum, text_max, threshold total *
    global_thr as a float).
    """
    H, text_seq, img_seq = block.shape
    block = _stage(np.asarray(block, dtype=np.float32), stage)
    hs = np.zeros(block.shape[1:], dtype=np.float32)
    for h in range(H):
        hs = (hs + block[h]).astype(np.float32)
    head_mean = _stage(hs / np.float32(H), stage)
    col = np.zeros(img_seq, dtype=np.float32)
    for c0 in range(0, text_seq, 32):
        part = np.zeros(img_seq, dtype=np.float32)
        for i in range(c0, min(text_seq, c0 + 32)):
            part = (part + head_mean[i]).astype(np.float32)
        col = (col + part).astype(np.float32)
    attn_sum = _stage(col, stage)
    text_max = head_mean.max(axis=0) if text_seq else np.full(img_seq, -np.inf, dtype=np.float32)
    t = np.float32(0)
    for t0 in range(0, img_seq, 32):
        ts = np.float32(0)
        for c in range(t0, min(img_seq, t0 + 32)):
            ts = np.float32(ts + attn_sum[c])
        t = np.float32(t + ts)
    total = _stage(np.float32(t), stage)
    thr = _stage(total * np.float32(global_thr), stage)[()]
    # torch compares a 16-bit tensor with a Python scalar after casting the scalar to the
    # tensor's dtype (line 62), so the individual threshold is rounded to the stage dtype too
    ithr = _stage(np.float32(individual_thr), stage)[()]
    drop = (attn_sum < thr) & (text_max < ithr)
    return np.nonzero(~drop)[0].astype(np.int64), attn_sum, text_max, float(thr)


def dual_attention_filter(attn: np.ndarray, v_token_start: int, img_seq: int, global_thr: float = 1.0,
                          individual_thr: float = 0.0, stage: str = "f32"):
    """Restates dual_attention_filter (qwen-eljrte/Qwen_Transformer/dual_attention_filter.py:6-103).

    attn [B, H, T, T] (batch 0 used).  block = attn[0, :, text rows, image columns] (lines
    37-43), then image_filter_block.  Returns (kept image-token indices ascending, text_seq,
    attn_sum, text_max, threshold total * global_thr as a float).
    """
    B, H, T, _ = attn.shape
    text_seq = T - img_seq - v_token_start
    img_beg, img_end = v_token_start, v_token_start + img_seq
    txt_beg, txt_end = img_end, img_end + text_seq
    block = np.asarray(attn[0, :, txt_beg:txt_end, img_beg:img_end], dtype=np.float32)
    kept, attn_sum, text_max, thr = image_filter_block(block, global_thr, individual_thr, stage)
    return kept, int(text_seq), attn_sum, text_max, thr
