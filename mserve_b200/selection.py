"""Drop-ins for the selection and sparse-attention functions of MServe's attention module.

Reference: qwen-eljrte/Qwen_Transformer/attention.py
  * compute_token_importance (532-588)  -> mskv_score + mskv_topk
  * sparse_sdpa_attention (591-641)     -> mskv_sparse_attention
and qwen-eljrte/Qwen_Transformer/dual_attention_filter.py
  * dual_attention_filter (6-103)       -> mskv_image_filter
  * repeat_kv (1701-1710)               -> same torch view/reshape (plumbing only; the
                                           kernels here never need repeated heads)

Beyond the reference signature, ``compute_token_importance`` takes keyword-only options for
the per-(sequence, KV head) selection with a recent window that the B200 path uses
(``per_kv_head=True``) and can leave the indices on the device (``return_device=True``).
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F

from . import ops

_METHODS = {"attention_score": 0, "norm": 1}


def repeat_kv(hidden_states: torch.Tensor, n_rep: int) -> torch.Tensor:
    """[B, Hkv, T, D] -> [B, Hkv*n_rep, T, D] (attention.py:1701-1710)."""
    batch, num_key_value_heads, slen, head_dim = hidden_states.shape
    if n_rep == 1:
        return hidden_states
    hidden_states = hidden_states[:, :, None, :, :].expand(batch, num_key_value_heads, n_rep, slen, head_dim)
    return hidden_states.reshape(batch, num_key_value_heads * n_rep, slen, head_dim)


def reference_top_k(T: int, top_k_ratio: float, min_tokens: int) -> int:
    """k = min(max(min_tokens, int(T * top_k_ratio)), T) (attention.py:567-569)."""
    return min(max(min_tokens, int(T * top_k_ratio)), T)


def head_scores(query: torch.Tensor, key: torch.Tensor, method: str = "attention_score",
                out: Optional[torch.Tensor] = None, lens: Optional[torch.Tensor] = None) -> torch.Tensor:
    """fp32 [B, Hk, T] importance per (sequence, KV head): GQA-summed q·k or ||k||.

    query [B, H, Q, D] (last query row used) or [B, H, D]; key [B, Hk, T, D] on the GPU.
    """
    if method not in _METHODS:
        raise ValueError(f"Unknown importance method: {method}")
    if key.dim() != 4 or not key.is_cuda:
        raise ValueError("key must be a CUDA tensor [B, Hk, T, D]")
    B, Hk, T, D = key.shape
    q = query[:, :, -1, :] if query.dim() == 4 else query
    if q.shape[0] != B or q.shape[-1] != D or q.shape[1] % Hk:
        raise ValueError(f"query {tuple(query.shape)} does not match key {tuple(key.shape)}")
    if key.stride(3) != 1:
        key = key.contiguous()
    if q.stride(-1) != 1:
        q = q.contiguous()
    if out is None:
        out = torch.empty(B, Hk, T, dtype=torch.float32, device=key.device)
    rows = ops.strided_rows(key, None, len_=lens, device=key.device)
    ops.score(q, rows, batch=B, kv_heads=Hk, max_tokens=T, out=out, method=_METHODS[method])
    return out


def compute_token_importance(query: torch.Tensor, key: torch.Tensor, method: str = "attention_score",
                             top_k_ratio: float = 0.3, min_tokens: int = 128, *,
                             per_kv_head: bool = False, top_k: Optional[int] = None, recent_window: int = 0,
                             return_device: bool = False, index_dtype: torch.dtype = torch.int64):
    """Indices of the tokens to keep (attention.py:532-588).

    Reference mode (default): scores are averaged over all query heads (key may hold the
    repeat_kv'd heads, as in the reference, or the KV heads themselves -- the result is the
    same), k = min(max(min_tokens, int(T*top_k_ratio)), T), and the result is a CPU int64
    tensor [k] for batch 1 (the reference's ``.squeeze(0)``) or [B, k].  Indices are returned
    in ascending order (the reference returns torch.topk's unsorted order; the set is the
    same, ties aside).

    per_kv_head=True: one selection per (sequence, KV head) over the GQA-summed scores:
    the top ``top_k`` (default: the reference's k rule) of [0, T - recent_window) plus the
    window [T - recent_window, T).  Returns (indices [B, Hk, K + R], counts int32 [B, Hk]),
    on the device.
    """
    if method not in _METHODS:
        raise ValueError(f"Unknown importance method: {method}")
    B, H = query.shape[0], query.shape[1]
    Hk, T = key.shape[1], key.shape[2]
    if H % Hk:
        raise ValueError("query heads must be a multiple of key heads")
    scores = head_scores(query, key, method)
    if per_kv_head:
        k = reference_top_k(T, top_k_ratio, min_tokens) if top_k is None else int(top_k)
        idx, counts = ops.topk(scores.view(B * Hk, T), top_k=k, recent=recent_window, rows_per_sel=1,
                               sel_per_batch=Hk, out_dtype=index_dtype)
        return idx.view(B, Hk, -1), counts.view(B, Hk)
    k = reference_top_k(T, top_k_ratio, min_tokens) if top_k is None else int(top_k)
    # mean over the H query heads: attention_score sums the Hk GQA-summed rows / H; norm
    # averages the Hk distinct key norms (each repeated H/Hk times in the reference).
    scale = 1.0 / H if method == "attention_score" else 1.0 / Hk
    idx, _ = ops.topk(scores.view(B * Hk, T), top_k=k, recent=0, rows_per_sel=Hk, sel_per_batch=1,
                      scale=scale, out_dtype=torch.int64)
    idx = idx[:, :k]
    if B == 1:
        idx = idx.squeeze(0)
    if return_device:
        return idx
    return idx.cpu().long()


def sparse_sdpa_attention(query: torch.Tensor, key_full: Optional[torch.Tensor], value_full: Optional[torch.Tensor],
                          key_sparse: torch.Tensor, value_sparse: torch.Tensor, sparse_indices: Optional[torch.Tensor],
                          attn_mask: Optional[torch.Tensor] = None, dropout_p: float = 0.0, is_causal: bool = False,
                          *, counts: Optional[torch.Tensor] = None) -> torch.Tensor:
    """softmax(q·K_sparseᵀ/sqrt(D))·V_sparse over the selected tokens (attention.py:591-641).

    Like the reference, key_full/value_full/sparse_indices/attn_mask/is_causal are accepted
    and unused.  key_sparse/value_sparse may hold the KV heads [B, Hk, S, D] (Hq % Hk == 0)
    instead of repeat_kv'd heads; ``counts`` [B, Hk] limits the rows of each head.
    dropout_p > 0 applies dropout to the output, as the reference does (attention.py:638-639).
    """
    ks, vs = key_sparse, value_sparse
    if ks.stride(3) != 1 or ks.stride(2) != ks.shape[3] or ks.stride(0) != ks.shape[1] * ks.stride(1):
        ks = ks.contiguous()
    if vs.stride() != ks.stride():
        vs = vs.contiguous()
        if vs.stride() != ks.stride():
            ks = ks.contiguous()
    out = ops.sparse_attention(query, ks, vs, counts=counts, scale=1.0 / math.sqrt(query.shape[-1]))
    if dropout_p > 0:
        out = F.dropout(out, p=dropout_p, training=True)
    return out


def dual_attention_filter(attn: torch.Tensor, v_token_start: int, img_seq: int, global_thr: float = 1.0,
                          individual_thr: float = 0.0, min_keep_ratio: float = 0.35, use_fp16: bool = False):
    """Image tokens kept by the prefill dual-threshold filter (dual_attention_filter.py:6-103).

    attn: [B, H, T, T] attention probabilities (batch 0 is used, as in the reference).  From the
    head-averaged text x image block, image token j is dropped when its column sum is below
    global_thr times the sum of all column sums and its column maximum is below
    individual_thr.  Returns (important_indices int64 [M] on attn's device, ascending,
    text_seq = T - img_seq - v_token_start).  min_keep_ratio is accepted and, as in the
    reference, not applied.  Each stage (head mean, column sums, total, threshold) is rounded to
    the block's dtype, fp16 when use_fp16 rounds an fp32 block first, as the reference's tensor
    arithmetic does; the sums accumulate in fp32.  individual_thr is rounded to that dtype too
    before the comparison, as torch casts a Python scalar to a tensor's dtype.
    """
    if attn.dim() != 4:
        raise AssertionError("attn must be [B, H, T, T]")
    B, H, T, _ = attn.shape
    if B < 1:
        raise AssertionError("attn has no batch")
    text_seq = T - img_seq - v_token_start
    idx, count = ops.image_filter(attn[0], img_start=v_token_start, img_seq=img_seq,
                                  text_start=v_token_start + img_seq, text_seq=text_seq, global_thr=global_thr,
                                  individual_thr=individual_thr,
                                  round_f16=bool(use_fp16) and attn.dtype == torch.float32)
    return idx[:int(count.item())], int(text_seq)

