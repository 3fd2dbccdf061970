"""KV heads sharded over the GPUs of one node.

One process per GPU; rank r holds the KV heads [r*Hl, (r+1)*Hl) of every sequence, Hl =
Hkv / world, in its own host store, and gathers them over its own host link.

* Per-(sequence, KV head) selection (the recent-window top-k) needs no exchange: each rank
  scores, selects, gathers and attends its own heads, and nothing crosses NVLink.
* The reference's shared selection -- one index set per sequence ranked by the mean over all
  query heads (qwen-eljrte/Qwen_Transformer/attention.py:558-572) -- needs every head's
  scores.  Each rank writes the GQA-summed fp32 score rows of its KV heads, [B, Hl, T]; one
  NCCL all-gather over NVLink lands every rank's rows in every rank's HBM as
  [world, B, Hl, T]; the top-k kernel then sums the Hkv rows of each sequence in global head
  order (its blocked row layout), which is the same fp32 sum, in the same order, as on one
  GPU holding all heads.  The selection is therefore identical on every rank and identical
  to the unsharded one.  The rows are all-gathered rather than all-reduced so that the
  summation order, and with it every tie, does not depend on the number of ranks.

The exchange is the only collective on the path, and it moves score rows (B*T*4 bytes per
head), never KV rows.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist

from . import ops


def head_shard(kv_heads: int, world: int, rank: int) -> Tuple[int, int]:
    """The KV heads [h0, h1) that `rank` of `world` holds (contiguous, equal shares)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if kv_heads % world:
        raise ValueError(f"{kv_heads} KV heads do not split evenly over {world} ranks")
    hl = kv_heads // world
    return rank * hl, (rank + 1) * hl


def exchange_head_scores(local: torch.Tensor, gathered: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather every rank's per-head score rows.

    local: contiguous [B, Hl, T]; gathered: contiguous [world, B, Hl, T] (rank-major, so the
    heads come in global order).  NCCL for CUDA tensors; any backend that implements
    all_gather_into_tensor on a dim-0 concatenated output (gloo on CPU tensors) works.
    """
    world = dist.get_world_size(group)
    if not local.is_contiguous() or not gathered.is_contiguous():
        raise ValueError("score buffers must be contiguous")
    if gathered.numel() != world * local.numel():
        raise ValueError(f"gathered holds {gathered.numel()} elements, expected {world} x {local.numel()}")
    if world == 1:                       # one rank holds every head: a device copy
        gathered.view_as(local).copy_(local)
        return gathered
    dist.all_gather_into_tensor(gathered.view(world * local.shape[0], *local.shape[1:]), local, group=group)
    return gathered


class SharedSelection:
    """Shared (per-sequence) selection over KV heads sharded across the ranks of `group`.

    The sharded counterpart of compute_token_importance's reference mode: scores averaged over
    all query heads, k = top_k per sequence, optionally plus a recent window.  Buffers are
    allocated once for `batch` sequences of up to `max_tokens` tokens.
    """

    def __init__(self, batch: int, kv_heads: int, q_heads: int, max_tokens: int, *, group=None,
                 device: Optional[torch.device] = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if q_heads % kv_heads:
            raise ValueError("query heads must be a multiple of KV heads")
        self.B, self.Hkv, self.Hq, self.T = batch, kv_heads, q_heads, max_tokens
        self.h0, self.h1 = head_shard(kv_heads, self.world, self.rank)
        self.Hl = self.h1 - self.h0
        self.G = q_heads // kv_heads
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.local = torch.empty(batch, self.Hl, max_tokens, dtype=torch.float32, device=self.device)
        self.gathered = torch.empty(self.world, batch, self.Hl, max_tokens, dtype=torch.float32,
                                    device=self.device)

    def q_heads_local(self) -> Tuple[int, int]:
        """The query heads [q0, q1) whose KV heads this rank holds."""
        return self.h0 * self.G, self.h1 * self.G

    def select(self, q_local: torch.Tensor, k_local: ops.RowsSpec, *, top_k: int, recent: int = 0,
               len_: Optional[torch.Tensor] = None, len_scalar: Optional[int] = None, method: int = 0,
               out: Optional[torch.Tensor] = None, counts: Optional[torch.Tensor] = None,
               out_dtype: torch.dtype = torch.int32):
        """One index set per sequence, the same on every rank.

        q_local: [B, Hl*G, D] (this rank's query heads); k_local: the keys of this rank's KV
        heads (ops.strided_rows / ops.paged_rows with Hl heads).  Returns (idx [B, K+R],
        counts int32 [B]).
        """
        T = self.T if len_scalar is None else int(len_scalar)
        ops.score(q_local, k_local, batch=self.B, kv_heads=self.Hl, max_tokens=T, out=self.local,
                  method=method)
        exchange_head_scores(self.local, self.gathered, self.group)
        scale = 1.0 / self.Hq if method == 0 else 1.0 / self.Hkv
        return ops.topk(self.gathered, top_k=top_k, recent=recent, len_=len_, len_scalar=T,
                        rows_per_sel=self.Hkv, sel_per_batch=1, scale=scale, out=out, counts=counts,
                        out_dtype=out_dtype, row_blocks=(self.world, self.B, self.Hl))
