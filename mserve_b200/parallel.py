"""KV heads sharded over the GPUs of one node.

One process per GPU; rank r holds the KV heads [r*Hl, (r+1)*Hl) of every sequence, Hl =
Hkv / world, in its own host store, and gathers them over its own host link.  With more ranks
than KV heads the sequences are split too (shard_plan): every (sequence, KV head) pair lives on
exactly one rank.  Host links differ in what they sustain when every GPU pulls at once, so the
sequences can be shared out by measured link rate (seq_split), and plan_for_links picks the
head-group count and the sequence shares that finish soonest for given per-rank rates.

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
head), never KV rows.  Two forms:
* "nccl": the score kernel writes this rank's rows, then an NCCL all-gather;
* "peer" (PeerExchange): the score kernel itself stores every row into every rank's buffer
  through CUDA IPC mappings (mskv_score_fanout), so the rows cross NVLink while the keys are
  still being read, and epoch flags in peer memory replace the collective.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib, ops


def head_shard(kv_heads: int, world: int, rank: int) -> Tuple[int, int]:
    """The KV heads [h0, h1) that `rank` of `world` holds (contiguous, equal shares)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if kv_heads % world:
        raise ValueError(f"{kv_heads} KV heads do not split evenly over {world} ranks")
    hl = kv_heads // world
    return rank * hl, (rank + 1) * hl


@dataclass(frozen=True)
class ShardPlan:
    """The (sequence, KV head) block of one rank when `world` ranks split one decode problem of
    `batch` sequences x `kv_heads` KV heads.  The KV heads are split first (head_groups =
    min(world, kv_heads) groups of kv_heads / head_groups heads); when there are more ranks than
    KV heads, the sequences are split as well (seq_groups = world / head_groups groups).  Rank r
    holds heads [h0, h1) of sequences [b0, b1) with head group r % head_groups and sequence
    group r // head_groups, so the ranks of one sequence group are consecutive and hold its
    heads in order -- the process group of a shared selection over those heads."""
    world: int
    rank: int
    head_groups: int
    seq_groups: int
    b0: int
    b1: int
    h0: int
    h1: int

    @property
    def seq_group(self) -> int:
        return self.rank // self.head_groups

    def group_ranks(self, seq_group: int):
        """Global ranks of one sequence group, in head order."""
        return list(range(seq_group * self.head_groups, (seq_group + 1) * self.head_groups))


def seq_split(batch: int, weights) -> list:
    """Sequences per sequence group for groups that move rows at the given relative rates: at
    least one each, the rest handed out one at a time to the group whose time (sequences / rate)
    grows least, which minimises the largest time.  Equal rates give an even split (ties go to
    the lower group)."""
    w = [float(x) for x in weights]
    if not w or any(not x > 0 for x in w):
        raise ValueError(f"sequence-group rates must be positive, got {weights}")
    if batch < len(w):
        raise ValueError(f"{batch} sequences cannot cover {len(w)} sequence groups")
    n = [1] * len(w)
    for _ in range(batch - len(w)):
        g = min(range(len(w)), key=lambda i: ((n[i] + 1) / w[i], i))
        n[g] += 1
    return n


def shard_plan(batch: int, kv_heads: int, world: int, rank: int, seq_weights=None,
               head_groups: Optional[int] = None) -> ShardPlan:
    """Splits batch x kv_heads (sequence, KV head) pairs over `world` ranks (see ShardPlan).

    The KV heads always split evenly, over head_groups groups (default min(world, kv_heads)).
    When there are more ranks than head groups the sequences are split too: evenly, or, with
    seq_weights (one relative rate per sequence group, e.g. the slowest measured host-link rate
    among the group's ranks), by seq_split so that groups on faster links take more sequences.
    Every rank must pass the same arguments."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    hg = min(world, kv_heads) if head_groups is None else int(head_groups)
    if hg <= 0 or kv_heads % hg or world % hg:
        raise ValueError(f"{world} ranks cannot split {kv_heads} KV heads evenly over {hg} head groups")
    sg = world // hg
    hl = kv_heads // hg
    hi, si = rank % hg, rank // hg
    if seq_weights is None or sg == 1:
        if batch % sg:
            raise ValueError(f"{world} ranks over {kv_heads} KV heads leave {sg} sequence groups, which do not "
                             f"split {batch} sequences evenly")
        bl = batch // sg
        b0, b1 = si * bl, (si + 1) * bl
    else:
        if len(seq_weights) != sg:
            raise ValueError(f"{len(seq_weights)} sequence-group weights for {sg} sequence groups")
        counts = seq_split(batch, seq_weights)
        b0 = sum(counts[:si])
        b1 = b0 + counts[si]
    return ShardPlan(world, rank, hg, sg, b0, b1, hi * hl, (hi + 1) * hl)


def plan_for_links(batch: int, kv_heads: int, world: int, rank: int, rates, min_gain: float = 0.03):
    """The split of batch x kv_heads (sequence, KV head) pairs of equal-length sequences over
    `world` ranks whose host links move `rates[r]` (e.g. GB/s, measured with all ranks copying at
    once).  Every head-group count hg that divides kv_heads and world is tried: sequence group g
    (ranks g*hg .. g*hg + hg - 1) moves at its slowest rank's rate, takes seq_split's share of the
    sequences (all of them with one group), and the group with the longest time sets the step.
    The default plan (hg = min(world, kv_heads), sequence groups weighted) is kept unless another
    hg is faster by more than min_gain.  Returns (plan, seq_weights or None, sequences per group,
    bound), bound being the job's rate in the units of `rates`.  Every rank must pass the same
    rates."""
    if len(rates) != world:
        raise ValueError(f"{len(rates)} link rates for {world} ranks")

    def evaluate(hg):
        sg = world // hg
        w = [min(rates[r] for r in range(g * hg, (g + 1) * hg)) for g in range(sg)]
        counts = seq_split(batch, w) if sg > 1 else [batch]
        step = max(n * (kv_heads // hg) / r for n, r in zip(counts, w))
        return (w if sg > 1 else None), counts, batch * kv_heads / step

    default = min(world, kv_heads)
    best = (default,) + evaluate(default)
    for hg in range(default - 1, 0, -1):
        if kv_heads % hg or world % hg or batch < world // hg:
            continue
        cand = (hg,) + evaluate(hg)
        if cand[3] > best[3] * (1.0 + min_gain):
            best = cand
    hg, weights, counts, bound = best
    return shard_plan(batch, kv_heads, world, rank, seq_weights=weights, head_groups=hg), weights, counts, bound


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


class PeerExchange:
    """Score rows of every rank stored straight into every rank's buffer by the score kernel.

    Each rank allocates (mskv_ipc_alloc) two buffers [world, B, Hl, T] fp32 -- the call's
    epoch e (1, 2, ...) uses parity e % 2 -- and an int64 flag array ready[2][world], and maps
    every other rank's through CUDA IPC.  One exchange (score()):
      1. the score kernel stores this rank's rows into block `rank` of parity p of every
         rank's buffer (its own directly, the others' over NVLink) and makes them
         system-visible;
      2. signal: ready[p][rank] = e in every rank's flags;
      3. wait until ready[p][s] reaches e for every rank s: the buffer is complete.
    The caller then reads the buffer (the top-k) on the same stream.  Two buffers make a
    separate "consumed" handshake unnecessary: a rank writes parity p again at epoch e + 2
    only after every rank signalled epoch e + 1, which each does after its stream finished
    reading epoch e.  Every wait is bounded (timeout_s); expiry sets the timeout status bit and
    lets the stream go on.  A wait that expired breaks the two-buffer argument (a lagging peer
    may still be writing into the buffer being read), so check_status(), which reads the
    status bits, marks the exchange unusable when it finds that bit: every later score() raises,
    and the exchange must be closed and created again.  Every rank must make the same sequence
    of calls.
    """

    def __init__(self, batch: int, local_heads: int, max_tokens: int, *, group=None,
                 device: Optional[torch.device] = None, timeout_s: float = 5.0, backend=None):
        # backend: the memory, flag and score operations (default: the CUDA library, ops)
        self.ops = backend if backend is not None else ops
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("the peer exchange spans at most 8 GPUs (one node)")
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.timeout_s = float(timeout_s)
        self.shape = (self.world, batch, local_heads, max_tokens)
        self.block = batch * local_heads * max_tokens            # elements of one rank's rows
        W = self.world
        self.buf, hb = self.ops.ipc_alloc(2 * W * self.block * 4)
        self.flags, hf = self.ops.ipc_alloc(2 * W * 8)
        got = [None] * W
        dist.all_gather_object(got, (hb, hf, self.shape), group=group)
        self.peer_buf: Dict[int, int] = {}
        self.peer_flags: Dict[int, int] = {}
        for r, (hbr, hfr, shape) in enumerate(got):
            if tuple(shape) != self.shape:
                raise ValueError(f"rank {r} exchanges {tuple(shape)}, this rank {self.shape}")
            if r == self.rank:
                self.peer_buf[r], self.peer_flags[r] = self.buf, self.flags
            else:
                self.peer_buf[r], self.peer_flags[r] = self.ops.ipc_open(hbr), self.ops.ipc_open(hfr)
        self.views = [self.ops.device_tensor(self.buf + p * W * self.block * 4, self.shape, torch.float32, self.device)
                      for p in (0, 1)]
        self.epoch = 0
        self.closed = False
        self.broken = False

    def check_status(self, what: str = "peer exchange") -> None:
        """Waits for this rank's stream, then raises RuntimeError if a kernel reported a status
        bit; a timed-out wait also marks the exchange unusable (see the class docstring)."""
        v = self.ops.take_status(self.device)
        if v & _lib.STATUS_TIMEOUT:
            self.broken = True
        if v:
            raise RuntimeError(f"{what}: {self.ops.describe_status(v)}")

    def _rows_at(self, r: int, parity: int) -> int:
        """Address of this rank's block in parity `parity` of rank r's buffer."""
        return self.peer_buf[r] + ((parity * self.world + self.rank) * self.block) * 4

    def score(self, q_local: torch.Tensor, k_local: ops.RowsSpec, *, max_tokens: int, method: int = 0) -> torch.Tensor:
        """Scores this rank's heads into every rank's buffer; returns this rank's complete
        [world, B, Hl, T] buffer of the new epoch, to be read on the current stream before the
        next call's score kernel (which follows on the same stream)."""
        if self.broken:
            raise RuntimeError("peer exchange unusable: a wait for another rank's scores timed out; "
                               "close() it and create a new one")
        if self.closed:
            raise RuntimeError("peer exchange is closed")
        W, e = self.world, self.epoch + 1
        p = e % 2
        _, B, Hl, T = self.shape
        self.ops.score(q_local, k_local, batch=B, kv_heads=Hl, max_tokens=max_tokens, out=self.views[p][self.rank],
                       method=method, peers=[self._rows_at(r, p) for r in range(W) if r != self.rank])
        self.ops.flag_signal([self.peer_flags[r] for r in range(W)], p * W + self.rank, e)
        self.ops.flag_wait(self.flags + p * W * 8, W, e, at_least=True, timeout_s=self.timeout_s, device=self.device)
        self.epoch = e
        return self.views[p]

    def close(self) -> None:
        """Unmaps the peers' memory and frees this rank's (collective: every rank calls it)."""
        if self.closed:
            return
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)           # nobody reads or writes the buffers any more
        for r in range(self.world):
            if r != self.rank:
                self.ops.ipc_close(self.peer_buf[r])
                self.ops.ipc_close(self.peer_flags[r])
        dist.barrier(group=self.group)           # every mapping of this rank's memory is closed
        self.ops.ipc_free(self.buf)
        self.ops.ipc_free(self.flags)
        self.closed = True


class SharedSelection:
    """Shared (per-sequence) selection over KV heads sharded across the ranks of `group`.

    The sharded counterpart of compute_token_importance's reference mode: scores averaged over
    all query heads, k = top_k per sequence, optionally plus a recent window.  Buffers are
    allocated once for `batch` sequences of up to `max_tokens` tokens.
    """

    def __init__(self, batch: int, kv_heads: int, q_heads: int, max_tokens: int, *, group=None,
                 device: Optional[torch.device] = None, exchange: str = "nccl", timeout_s: float = 5.0):
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
        if exchange not in ("nccl", "peer"):
            raise ValueError("exchange must be 'nccl' or 'peer'")
        self.exchange = exchange
        self.peer = None
        if exchange == "peer":
            self.peer = PeerExchange(batch, self.Hl, max_tokens, group=group, device=self.device,
                                     timeout_s=timeout_s)
        else:
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
        if self.peer is not None:
            gathered = self.peer.score(q_local, k_local, max_tokens=T, method=method)
        else:
            ops.score(q_local, k_local, batch=self.B, kv_heads=self.Hl, max_tokens=T, out=self.local,
                      method=method)
            gathered = exchange_head_scores(self.local, self.gathered, self.group)
        scale = 1.0 / self.Hq if method == 0 else 1.0 / self.Hkv
        res = ops.topk(gathered, top_k=top_k, recent=recent, len_=len_, len_scalar=T,
                       rows_per_sel=self.Hkv, sel_per_batch=1, scale=scale, out=out, counts=counts,
                       out_dtype=out_dtype, row_blocks=(self.world, self.B, self.Hl))
        return res

    def check_status(self, what: str = "shared selection") -> None:
        """Raises RuntimeError if a kernel of this rank reported a status bit (synchronising); with
        exchange='peer' a timed-out wait leaves the selection unusable until it is recreated."""
        if self.peer is not None:
            self.peer.check_status(what)
        else:
            ops.check_status(self.device, what)

    def close(self) -> None:
        """Releases the peer exchange's memory (collective with exchange='peer')."""
        if self.peer is not None:
            self.peer.close()
