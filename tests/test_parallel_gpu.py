"""Head-sharded shared selection on the GPU.

* Ranks emulated on one GPU: each "rank" scores its own KV heads with mskv_score, the rows are
  stacked rank-major (what the NCCL all-gather produces) and mskv_topk sums them through the
  blocked row layout.  Scores and selections must be bit-identical to the unsharded launch,
  and the selection must match the oracle's ranking of the GPU scores.
* Real ranks (two or more GPUs): SharedSelection on NCCL, one process per GPU, against the
  unsharded selection computed on each rank's own GPU.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import kv_oracle as ko

pytestmark = pytest.mark.gpu


def _case(seed, B, Hq, Hkv, T, D, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, D, generator=g).to(dtype)
    k = torch.randn(B, Hkv, T, D, generator=g).to(dtype)
    return q, k


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("method", [0, 1])
def test_emulated_ranks_bit_identical(built_lib, world, method):
    from mserve_b200 import ops
    B, Hq, Hkv, T, D, K, R = 3, 40, 8, 5000, 128, 700, 64
    q, k = _case(world * 10 + method, B, Hq, Hkv, T, D)
    dev = torch.device("cuda")
    q, k = q.to(dev), k.to(dev)
    G, Hl = Hq // Hkv, Hkv // world
    full = torch.empty(B, Hkv, T, device=dev)
    ops.score(q, ops.strided_rows(k), batch=B, kv_heads=Hkv, max_tokens=T, out=full, method=method)
    scale = 1.0 / Hq if method == 0 else 1.0 / Hkv
    ref_idx, ref_cnt = ops.topk(full, top_k=K, recent=R, rows_per_sel=Hkv, scale=scale)
    gathered = torch.empty(world, B, Hl, T, device=dev)
    for r in range(world):
        h0, h1 = r * Hl, (r + 1) * Hl
        ops.score(q[:, h0 * G:h1 * G].contiguous(), ops.strided_rows(k[:, h0:h1]), batch=B, kv_heads=Hl,
                  max_tokens=T, out=gathered[r], method=method)
    # per-head rows: bit-identical to the unsharded launch
    assert torch.equal(gathered.permute(1, 0, 2, 3).reshape(B, Hkv, T), full)
    idx, cnt = ops.topk(gathered, top_k=K, recent=R, rows_per_sel=Hkv, scale=scale,
                        row_blocks=(world, B, Hl))
    assert torch.equal(cnt, ref_cnt)
    assert torch.equal(idx, ref_idx)
    # and the oracle's ranking of the same fp32 rows
    sel, rc = ko.select_topk_window(full.view(B * Hkv, T).cpu().numpy(), top_k=K, recent=R, rows_per_sel=Hkv,
                                    scale=np.float32(scale))
    got, gc = idx.cpu().numpy(), cnt.cpu().numpy()
    np.testing.assert_array_equal(gc, rc)
    for b in range(B):
        np.testing.assert_array_equal(got[b, :gc[b]], sel[b])


def test_blocked_layout_ragged_lengths(built_lib):
    """Per-sequence lengths and top-k with the blocked layout (cluster path and large-T path)."""
    from mserve_b200 import ops
    dev = torch.device("cuda")
    for T in (3000, 140000):
        world, B, Hl = 2, 2, 2
        g = torch.Generator().manual_seed(T)
        rows = torch.randn(world, B, Hl, T, generator=g).to(dev)
        lens = torch.tensor([T, T // 3], dtype=torch.int32, device=dev)
        tk = torch.tensor([T // 10, 5], dtype=torch.int32, device=dev)
        idx, cnt = ops.topk(rows, top_k=tk, recent=7, len_=lens, rows_per_sel=world * Hl, scale=0.25,
                            row_blocks=(world, B, Hl))
        plain = rows.permute(1, 0, 2, 3).reshape(B * world * Hl, T).contiguous()
        ref_idx, ref_cnt = ops.topk(plain, top_k=tk, recent=7, len_=lens, rows_per_sel=world * Hl, scale=0.25)
        assert torch.equal(cnt, ref_cnt)
        for b in range(B):
            c = int(cnt[b])
            assert torch.equal(idx[b, :c], ref_idx[b, :c])


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from mserve_b200 import ops, parallel
        B, Hq, Hkv, T, D, K, R = 4, 40, 8, 32768, 128, 4096, 256
        q, k = _case(5, B, Hq, Hkv, T, D)                   # same data on every rank
        q, k = q.to(dev), k.to(dev)
        sel = parallel.SharedSelection(B, Hkv, Hq, T, device=dev)
        q0, q1 = sel.q_heads_local()
        idx, cnt = sel.select(q[:, q0:q1].contiguous(), ops.strided_rows(k[:, sel.h0:sel.h1]), top_k=K, recent=R)
        full = torch.empty(B, Hkv, T, device=dev)
        ops.score(q, ops.strided_rows(k), batch=B, kv_heads=Hkv, max_tokens=T, out=full)
        ref_idx, ref_cnt = ops.topk(full, top_k=K, recent=R, rows_per_sel=Hkv, scale=1.0 / Hq)
        torch.cuda.synchronize(dev)
        assert torch.equal(cnt, ref_cnt), f"rank {rank}: counts differ"
        assert torch.equal(idx, ref_idx), f"rank {rank}: selection differs from the unsharded one"
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_shared_selection_nccl(built_lib):
    world = 2
    mp.start_processes(_nccl_worker, args=(world, _free_port()), nprocs=world, join=True, start_method="spawn")


def test_score_fanout_writes_every_copy(built_lib):
    """mskv_score_fanout stores each score into the extra copies too (here two more device
    buffers of this GPU standing in for peers): all copies bit-identical to mskv_score."""
    from mserve_b200 import ops
    B, Hq, Hkv, T, D = 3, 16, 4, 3000, 128
    q, k = _case(21, B, Hq, Hkv, T, D)
    dev = torch.device("cuda")
    q, k = q.to(dev), k.to(dev)
    ref = torch.empty(B, Hkv, T, device=dev)
    ops.score(q, ops.strided_rows(k), batch=B, kv_heads=Hkv, max_tokens=T, out=ref)
    outs = [torch.full((B, Hkv, T), float("nan"), device=dev) for _ in range(3)]
    ops.score(q, ops.strided_rows(k), batch=B, kv_heads=Hkv, max_tokens=T, out=outs[0],
              peers=[outs[1].data_ptr(), outs[2].data_ptr()])
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o, ref)
    with pytest.raises(RuntimeError):
        ops.score(q, ops.strided_rows(k), batch=B, kv_heads=Hkv, max_tokens=T, out=outs[0], peers=[0])


def test_flag_wait_times_out_and_reports(built_lib):
    """A wait on a flag that nothing sets ends after its time limit with the timeout status
    (the stream goes on; check_status raises); a flag already set passes at once."""
    from mserve_b200 import ops
    dev = torch.device("cuda")
    ptr, _ = ops.ipc_alloc(64)
    try:
        flags = ops.device_tensor(ptr, (8,), torch.int64, dev)
        ops.flag_signal([ptr], 3, 7)
        ops.flag_wait(ptr + 3 * 8, 1, 7, timeout_s=0.05, device=dev)
        ops.flag_wait(ptr + 3 * 8, 1, 5, at_least=True, timeout_s=0.05, device=dev)
        ops.check_status(dev, "flag set")
        assert int(flags[3].item()) == 7
        ops.flag_wait(ptr + 4 * 8, 2, 1, timeout_s=0.05, device=dev)     # nothing sets flags 4, 5
        with pytest.raises(RuntimeError, match="timed out"):
            ops.check_status(dev, "flag never set")
    finally:
        torch.cuda.synchronize()
        ops.ipc_free(ptr)


def _single_rank(fn):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(_free_port())
    dev = torch.device("cuda", torch.cuda.current_device())
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        fn(dev)
    finally:
        dist.destroy_process_group()


def test_peer_exchange_one_rank_epochs(built_lib):
    """SharedSelection with the peer exchange on one rank: five successive selections (both
    buffer parities) equal the NCCL form's."""
    from mserve_b200 import ops, parallel

    def body(dev):
        B, Hq, Hkv, T, D, K, R = 4, 40, 8, 6000, 128, 500, 32
        sel_p = parallel.SharedSelection(B, Hkv, Hq, T, device=dev, exchange="peer")
        sel_n = parallel.SharedSelection(B, Hkv, Hq, T, device=dev)
        try:
            for step in range(5):
                q, k = _case(40 + step, B, Hq, Hkv, T, D)
                q, k = q.to(dev), k.to(dev)
                a = sel_p.select(q, ops.strided_rows(k), top_k=K, recent=R)
                b = sel_n.select(q, ops.strided_rows(k), top_k=K, recent=R)
                torch.cuda.synchronize(dev)
                assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1]), f"step {step}"
            ops.check_status(dev, "peer exchange")
            assert sel_p.peer.epoch == 5
        finally:
            sel_p.close()

    _single_rank(body)


def _peer_worker(rank, world, port):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    sel = None
    try:
        from mserve_b200 import ops, parallel
        B, Hq, Hkv, T, D, K, R = 4, 40, 8, 32768, 128, 4096, 256
        sel = parallel.SharedSelection(B, Hkv, Hq, T, device=dev, exchange="peer", timeout_s=5.0)
        q0, q1 = sel.q_heads_local()
        for step in range(4):
            q, k = _case(60 + step, B, Hq, Hkv, T, D)           # same data on every rank
            q, k = q.to(dev), k.to(dev)
            idx, cnt = sel.select(q[:, q0:q1].contiguous(), ops.strided_rows(k[:, sel.h0:sel.h1]), top_k=K, recent=R)
            full = torch.empty(B, Hkv, T, device=dev)
            ops.score(q, ops.strided_rows(k), batch=B, kv_heads=Hkv, max_tokens=T, out=full)
            ref_idx, ref_cnt = ops.topk(full, top_k=K, recent=R, rows_per_sel=Hkv, scale=1.0 / Hq)
            torch.cuda.synchronize(dev)
            ops.check_status(dev, f"rank {rank} step {step}")
            assert torch.equal(cnt, ref_cnt), f"rank {rank} step {step}: counts differ"
            assert torch.equal(idx, ref_idx), f"rank {rank} step {step}: selection differs from the unsharded one"
        dist.barrier()
    finally:
        if sel is not None:
            sel.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_shared_selection_peer_exchange(built_lib):
    """Two ranks, the score rows stored into each other's buffers by the score kernel."""
    world = 2
    mp.start_processes(_peer_worker, args=(world, _free_port()), nprocs=world, join=True, start_method="spawn")
