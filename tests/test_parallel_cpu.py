"""Head-sharded shared selection: the host logic on gloo ranks (CPU, world sizes 2 and 4).

Each rank computes the GQA-summed score rows of its own KV heads with the oracle, the rows are
exchanged with mserve_b200.parallel.exchange_head_scores, and the blocked row layout that
mserve_b200.parallel hands to the top-k kernel (ops.blocked_layout) is walked here the way the
kernel walks it.  Every sequence must see its Hkv rows in global head order, bit for bit, and
the oracle's selection over them must equal the unsharded selection.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import kv_oracle as ko


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(seed: int, B=3, Hq=16, Hkv=4, T=257, D=32):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, Hq, D)).astype(np.float32)
    k = rng.standard_normal((B, Hkv, T, D)).astype(np.float32)
    return q, k


def _rows_of_selection(flat: np.ndarray, j: int, rows: int, layout, row_len: int) -> np.ndarray:
    """Rows r = 0..rows-1 of selection j, addressed as mskv_topk addresses them."""
    sel_stride, row_block, block_stride = layout
    out = []
    for r in range(rows):
        off = j * sel_stride + (r // row_block) * block_stride + (r % row_block) * row_len
        out.append(flat[off:off + row_len])
    return np.stack(out)


def _worker(rank, world, port, seed, top_k, recent):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from mserve_b200 import ops, parallel
        q, k = _case(seed)
        B, Hq, _ = q.shape
        Hkv, T = k.shape[1], k.shape[2]
        G = Hq // Hkv
        full = ko.gqa_scores(q, k).astype(np.float32)                  # [B, Hkv, T], all heads
        h0, h1 = parallel.head_shard(Hkv, world, rank)
        Hl = h1 - h0
        local = ko.gqa_scores(q[:, h0 * G:h1 * G], k[:, h0:h1]).astype(np.float32)
        assert np.array_equal(local, full[:, h0:h1])                    # heads are independent
        gathered = torch.empty(world, B, Hl, T)
        parallel.exchange_head_scores(torch.from_numpy(np.ascontiguousarray(local)), gathered)
        layout = ops.blocked_layout(world, B, Hl, T)
        flat = gathered.numpy().reshape(-1)
        for b in range(B):
            rows = _rows_of_selection(flat, b, Hkv, layout, T)
            assert np.array_equal(rows, full[b]), f"rank {rank}: rows of sequence {b} out of head order"
        # the selection over the exchanged rows equals the unsharded one
        regathered = np.stack([_rows_of_selection(flat, b, Hkv, layout, T) for b in range(B)]).reshape(B * Hkv, T)
        sel_s, cnt_s = ko.select_topk_window(regathered, top_k=top_k, recent=recent, rows_per_sel=Hkv,
                                             scale=np.float32(1.0 / Hq))
        sel_f, cnt_f = ko.select_topk_window(full.reshape(B * Hkv, T), top_k=top_k, recent=recent,
                                             rows_per_sel=Hkv, scale=np.float32(1.0 / Hq))
        assert list(cnt_s) == list(cnt_f)
        for a, b_ in zip(sel_s, sel_f):
            assert np.array_equal(a, b_)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_exchange_matches_unsharded(world):
    port = _free_port()
    mp.start_processes(_worker, args=(world, port, 17 + world, 40, 16), nprocs=world, join=True,
                       start_method="spawn")


def test_head_shard_splits():
    from mserve_b200 import parallel
    assert [parallel.head_shard(8, 4, r) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    assert parallel.head_shard(8, 1, 0) == (0, 8)
    with pytest.raises(ValueError):
        parallel.head_shard(4, 8, 0)          # fewer heads than ranks
    with pytest.raises(ValueError):
        parallel.head_shard(8, 2, 2)          # rank out of range


def test_blocked_layout_single_block_is_plain_rows():
    from mserve_b200 import ops
    # one block: row r of selection j at (j*R + r) * T -- the unsharded [B, Hkv, T] layout
    sel_stride, row_block, block_stride = ops.blocked_layout(1, 5, 4, 100)
    assert (sel_stride, row_block) == (400, 4)
    for j in range(5):
        for r in range(4):
            assert j * sel_stride + (r // row_block) * block_stride + (r % row_block) * 100 == (j * 4 + r) * 100


class _SharedMemoryBackend:
    """The peer exchange's memory, flag and score operations on the CPU, for its host logic:
    shared-memory segments stand in for IPC device memory (an "address" is a registered base
    plus an offset), flag waits poll the segment from the host, and the score is the oracle's
    GQA-summed rows.  Every store into a peer goes through the same address arithmetic that
    the CUDA path hands to the kernels."""

    def __init__(self, rank):
        self.rank = rank
        self.segs = {}                  # base -> (SharedMemory, size)
        self.next = (rank + 1) << 40
        self.status = 0                 # the device status word

    def _register(self, shm, size):
        base = self.next
        self.next += 1 << 32
        self.segs[base] = (shm, size)
        return base

    def _view(self, addr, count, dtype):
        for base, (shm, size) in self.segs.items():
            if base <= addr < base + size:
                off = addr - base
                assert off + count * np.dtype(dtype).itemsize <= size, "access beyond the allocation"
                return np.ndarray((count,), dtype=dtype, buffer=shm.buf, offset=off)
        raise AssertionError(f"address {addr:#x} is in no allocation")

    def ipc_alloc(self, nbytes):
        from multiprocessing import shared_memory
        shm = shared_memory.SharedMemory(create=True, size=nbytes)
        np.ndarray((nbytes,), dtype=np.uint8, buffer=shm.buf)[:] = 0
        return self._register(shm, nbytes), shm.name.encode()

    def ipc_open(self, handle):
        from multiprocessing import shared_memory
        shm = shared_memory.SharedMemory(name=handle.decode())
        return self._register(shm, shm.size)

    def ipc_close(self, ptr):
        shm, _ = self.segs.pop(ptr)
        shm.close()

    def ipc_free(self, ptr):
        shm, _ = self.segs.pop(ptr)
        shm.close()
        shm.unlink()

    def device_tensor(self, ptr, shape, dtype, device):
        n = int(np.prod(shape))
        return torch.from_numpy(self._view(ptr, n, np.float32).reshape(shape))

    def score(self, q, k, *, batch, kv_heads, max_tokens, out, method=0, peers=()):
        rows = ko.gqa_scores(q, k).astype(np.float32)[:, :, :max_tokens]
        out[:, :, :max_tokens] = torch.from_numpy(rows)
        n = batch * kv_heads * out.shape[2]
        for p in peers:
            self._view(p, n, np.float32).reshape(out.shape)[:, :, :max_tokens] = rows

    def flag_signal(self, flag_arrays, index, value, stream=None):
        for f in flag_arrays:
            self._view(f + index * 8, 1, np.int64)[0] = value

    def flag_wait(self, flags, count, value, *, at_least=False, timeout_s=1.0, device=None, stream=None):
        import time
        v = self._view(flags, count, np.int64)
        t0 = time.monotonic()
        while not all((x >= value) if at_least else (x == value) for x in v):
            if time.monotonic() - t0 > timeout_s:
                self.status |= 0x8      # as the device wait does: a status bit, and go on
                return
            time.sleep(0.0005)

    def take_status(self, device):
        v, self.status = self.status, 0
        return v

    def describe_status(self, v):
        return f"status 0x{v:x}"


def _peer_worker(rank, world, port, epochs):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from mserve_b200 import parallel
        B, Hq, Hkv, T, D = 2, 16, 8, 100, 16
        Hl = Hkv // world
        G = Hq // Hkv
        be = _SharedMemoryBackend(rank)
        ex = parallel.PeerExchange(B, Hl, T, device=torch.device("cpu"), timeout_s=20.0, backend=be)
        rng = np.random.default_rng(rank)
        for e in range(1, epochs + 1):
            q, k = _case(100 + e, B=B, Hq=Hq, Hkv=Hkv, T=T, D=D)       # the same on every rank
            h0, h1 = rank * Hl, (rank + 1) * Hl
            if rng.random() < 0.5:                                    # ranks drift apart
                import time
                time.sleep(rng.random() * 0.02)
            view = ex.score(q[:, h0 * G:h1 * G], k[:, h0:h1], max_tokens=T)
            if rng.random() < 0.5:                                    # a slow reader of the buffer
                import time
                time.sleep(rng.random() * 0.02)
            got = view.numpy().copy()
            want = ko.gqa_scores(q, k).astype(np.float32).reshape(B, world, Hl, T).transpose(1, 0, 2, 3)
            np.testing.assert_array_equal(got, want, err_msg=f"rank {rank} epoch {e}")
            assert ex.epoch == e
        ex.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_peer_exchange_protocol(world):
    """PeerExchange's buffer parities, block offsets and epoch flags on gloo ranks: every
    epoch's gathered buffer holds every rank's rows of that epoch (none of another epoch),
    while ranks drift apart and read their buffers late by random delays."""
    mp.start_processes(_peer_worker, args=(world, _free_port(), 7), nprocs=world, join=True, start_method="spawn")


def _timeout_worker(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from mserve_b200 import parallel
        B, Hq, Hkv, T, D = 2, 8, 4, 50, 16
        Hl, G = Hkv // world, Hq // Hkv
        be = _SharedMemoryBackend(rank)
        ex = parallel.PeerExchange(B, Hl, T, device=torch.device("cpu"), timeout_s=0.3, backend=be)
        q, k = _case(7, B=B, Hq=Hq, Hkv=Hkv, T=T, D=D)
        h0, h1 = rank * Hl, (rank + 1) * Hl
        ex.score(q[:, h0 * G:h1 * G], k[:, h0:h1], max_tokens=T)           # epoch 1: every rank
        ex.check_status()
        if rank == 0:                                                       # epoch 2: rank 1 never joins
            ex.score(q[:, h0 * G:h1 * G], k[:, h0:h1], max_tokens=T)
            with pytest.raises(RuntimeError, match="0x8"):
                ex.check_status()
            assert ex.broken
            with pytest.raises(RuntimeError, match="unusable"):
                ex.score(q[:, h0 * G:h1 * G], k[:, h0:h1], max_tokens=T)
        else:
            assert not ex.broken
        ex.close()
    finally:
        dist.destroy_process_group()


def test_peer_exchange_timeout_leaves_it_unusable():
    """A rank that never joins an epoch: the other rank's bounded wait expires, check_status()
    raises on the timeout bit and every later score() refuses to run until the exchange is
    recreated (a lagging peer could still write into the buffer being read)."""
    mp.start_processes(_timeout_worker, args=(2, _free_port()), nprocs=2, join=True, start_method="spawn")


@pytest.mark.parametrize("B,Hkv,world", [(8, 4, 1), (8, 4, 2), (8, 4, 4), (8, 4, 8), (16, 8, 8), (32, 8, 4),
                                         (2, 1, 2)])
def test_shard_plan_covers_every_pair_once(B, Hkv, world):
    """Every (sequence, KV head) pair on exactly one rank; heads split before sequences; the
    ranks of a sequence group are consecutive and hold its heads in order."""
    from mserve_b200.parallel import shard_plan
    owner = {}
    for r in range(world):
        p = shard_plan(B, Hkv, world, r)
        assert p.head_groups == min(world, Hkv) and p.head_groups * p.seq_groups == world
        assert (p.b1 - p.b0) * (p.h1 - p.h0) * world == B * Hkv
        ranks = p.group_ranks(p.seq_group)
        assert r in ranks and ranks == sorted(ranks)
        assert [shard_plan(B, Hkv, world, q).h0 for q in ranks] == sorted(shard_plan(B, Hkv, world, q).h0 for q in ranks)
        for b in range(p.b0, p.b1):
            for h in range(p.h0, p.h1):
                assert (b, h) not in owner
                owner[(b, h)] = r
    assert len(owner) == B * Hkv


def test_shard_plan_rejects_uneven_splits():
    from mserve_b200.parallel import shard_plan
    with pytest.raises(ValueError):
        shard_plan(8, 4, 3, 0)          # 3 ranks over 4 heads
    with pytest.raises(ValueError):
        shard_plan(7, 4, 8, 0)          # 8 ranks over 4 heads: 2 sequence groups of 7 sequences
    with pytest.raises(ValueError):
        shard_plan(8, 4, 8, 8)


def test_seq_split_minimises_the_slowest_group():
    """Sequences per sequence group by link rate: equal rates give the even split, unequal rates
    the integer split whose largest sequences / rate is smallest (checked against every split)."""
    import itertools
    from mserve_b200.parallel import seq_split
    assert seq_split(8, [55.5, 55.4]) == [4, 4]
    assert seq_split(8, [1.0, 1.0, 1.0, 1.0]) == [2, 2, 2, 2]
    assert seq_split(8, [23.1, 35.1]) == [3, 5]
    for B, rates in [(8, [23.1, 35.1]), (9, [10.0, 20.0, 30.0]), (16, [5.0, 7.0, 11.0, 13.0]), (3, [1.0, 9.0, 2.0])]:
        got = seq_split(B, rates)
        assert sum(got) == B and min(got) >= 1
        best = min(max(n / r for n, r in zip(c, rates))
                   for c in itertools.product(range(1, B + 1), repeat=len(rates)) if sum(c) == B)
        assert max(n / r for n, r in zip(got, rates)) == pytest.approx(best)
    with pytest.raises(ValueError):
        seq_split(1, [1.0, 1.0])
    with pytest.raises(ValueError):
        seq_split(8, [1.0, 0.0])


@pytest.mark.parametrize("rates", [[23.1, 35.1], [35.1, 23.1], [30.0, 30.0]])
def test_weighted_shard_plan_covers_every_pair_once(rates):
    """With per-sequence-group weights every (sequence, KV head) pair is still on exactly one rank,
    and the ranks of a sequence group hold the same sequences (the shared selection's groups)."""
    from mserve_b200.parallel import seq_split, shard_plan
    B, Hkv, world = 8, 4, 8
    counts = seq_split(B, rates)
    owner = {}
    for r in range(world):
        p = shard_plan(B, Hkv, world, r, seq_weights=rates)
        assert p.b1 - p.b0 == counts[p.seq_group]
        for q in p.group_ranks(p.seq_group):
            o = shard_plan(B, Hkv, world, q, seq_weights=rates)
            assert (o.b0, o.b1) == (p.b0, p.b1)
        for b in range(p.b0, p.b1):
            for h in range(p.h0, p.h1):
                assert (b, h) not in owner
                owner[(b, h)] = r
    assert len(owner) == B * Hkv
    # one sequence group: the weights change nothing
    assert shard_plan(8, 4, 4, 1, seq_weights=[9.0]) == shard_plan(8, 4, 4, 1)
    with pytest.raises(ValueError):
        shard_plan(B, Hkv, world, 0, seq_weights=[1.0, 2.0, 3.0])


def test_plan_for_links_picks_head_groups_by_link_rates():
    """Equal links keep the default plan; uneven links move to fewer head groups only when the
    bound improves by more than 3%; every (sequence, KV head) pair stays on exactly one rank and
    the ranks of a sequence group hold the same sequences."""
    from mserve_b200.parallel import plan_for_links, shard_plan
    slow_fast = [23.4, 23.4, 23.5, 23.5, 35.9, 36.2, 35.9, 35.8]
    cases = [  # batch, kv heads, world, rates, expected head groups, sequences per group
        (16, 8, 8, [30.0] * 8, 8, [16]),
        (16, 8, 8, slow_fast, 4, [6, 10]),
        (8, 4, 8, slow_fast, 4, [3, 5]),
        (8, 4, 4, [23.0, 23.0, 36.0, 36.0], 2, [3, 5]),
        (8, 4, 4, [28.7, 28.5, 28.9, 28.8], 4, [8]),
        (8, 4, 2, [55.5, 55.4], 2, [8]),
    ]
    for B, H, world, rates, hg, counts in cases:
        owner = {}
        bounds = set()
        for r in range(world):
            plan, w, c, bound = plan_for_links(B, H, world, r, rates)
            assert plan.head_groups == hg and c == counts, (B, H, world, rates, plan, c)
            assert (w is None) == (len(counts) == 1)
            bounds.add(round(bound, 9))
            for q in plan.group_ranks(plan.seq_group):
                o = plan_for_links(B, H, world, q, rates)[0]
                assert (o.b0, o.b1) == (plan.b0, plan.b1)
            for b in range(plan.b0, plan.b1):
                for h in range(plan.h0, plan.h1):
                    assert (b, h) not in owner
                    owner[(b, h)] = r
        assert len(owner) == B * H and len(bounds) == 1
    # the default plan's bound is world x the slowest rate for equal shares
    _, _, _, bound = plan_for_links(16, 8, 8, 0, [30.0] * 8)
    assert bound == pytest.approx(240.0)
    assert shard_plan(16, 8, 8, 0, head_groups=4, seq_weights=[1.0, 1.0]).b1 == 8
    with pytest.raises(ValueError):
        plan_for_links(8, 4, 8, 0, [1.0] * 4)
