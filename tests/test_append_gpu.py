"""Parity of the append / write-back path (mskv_copy_rows) with the oracle and the reference.

Bit-exact: the CPUKVCache drop-in reproduces the reference's cat + keep-last-max_len host
cache (qwen-eljrte/Qwen_Transformer/kv_cache.py:718-765, golden vectors from the reference's
own append_new) with in-place ring writes; paged append and page write-back match the oracle.
"""
import numpy as np
import pytest
import torch

from conftest import from_bits, to_numpy_bits
from oracle import kv_oracle as ko

pytestmark = pytest.mark.gpu


def test_cpukvcache_append_matches_reference_golden(built_lib, golden):
    from mserve_b200.kv_cache import CPUKVCache
    max_len = int(golden["append/max_len"])
    cache = CPUKVCache(num_layers=2, max_len=max_len)
    for i in range(7):
        kn = from_bits(golden[f"append/step{i}/k_new"], torch.bfloat16).cuda()
        vn = from_bits(golden[f"append/step{i}/v_new"], torch.bfloat16).cuda()
        assert cache.submit_append(1, kn, vn)
        k, v, seq_len, ver = cache.get_snapshot(1)
        exp_len, exp_ver = [int(x) for x in golden[f"append/step{i}/meta"]]
        assert (seq_len, ver) == (exp_len, exp_ver)
        np.testing.assert_array_equal(to_numpy_bits(k), golden[f"append/step{i}/k"].view(np.int16))
        np.testing.assert_array_equal(to_numpy_bits(v), golden[f"append/step{i}/v"].view(np.int16))
        assert k.is_pinned()
    # the gather reads the wrapped ring in logical order
    idx = torch.from_numpy(golden["sparse/idx"])
    k_sel, v_sel, ev = cache.get_sparse_async_uva(1, torch.device("cuda"), idx)
    ev.synchronize()
    kk, vv, _, _ = cache.get_snapshot(1)
    ek, evv = ko.index_select_gather(to_numpy_bits(kk), to_numpy_bits(vv), idx.numpy())
    np.testing.assert_array_equal(to_numpy_bits(k_sel), ek)
    np.testing.assert_array_equal(to_numpy_bits(v_sel), evv)
    with pytest.raises(RuntimeError, match="out of range"):
        cache.get_sparse_async_uva(1, torch.device("cuda"), torch.tensor([max_len]))
    cache.shutdown()


def test_cpukvcache_ring_random_appends(built_lib):
    """Random append sizes (including > max_len at once) against the oracle's cat_truncate."""
    from mserve_b200.kv_cache import CPUKVCache
    g = torch.Generator().manual_seed(4)
    max_len = 100
    cache = CPUKVCache(num_layers=1, max_len=max_len)
    ok = ov = None
    for step in range(25):
        n = int(torch.randint(1, 130, (1,), generator=g))
        kn = torch.randn(2, 3, n, 128, generator=g).to(torch.bfloat16)
        vn = torch.randn(2, 3, n, 128, generator=g).to(torch.bfloat16)
        src_dev = step % 3 != 0            # also rows that already live on the host
        assert cache.submit_append(0, kn.cuda() if src_dev else kn, vn.cuda() if src_dev else vn)
        ok, ov = ko.cat_truncate(ok, ov, to_numpy_bits(kn), to_numpy_bits(vn), max_len)
        k, v, L, _ = cache.get_snapshot(0)
        assert L == ok.shape[2]
        np.testing.assert_array_equal(to_numpy_bits(k), ok)
        np.testing.assert_array_equal(to_numpy_bits(v), ov)


def test_cpukvcache_queue_bound_and_get_async(built_lib):
    from mserve_b200.kv_cache import CPUKVCache
    cache = CPUKVCache(num_layers=2, max_len=64, queue_maxsize=1)
    kn = torch.randn(1, 2, 10, 64).to(torch.bfloat16).cuda()
    assert cache.submit_append(0, kn, kn)
    torch.cuda.synchronize()
    assert cache.submit_append(0, kn, kn, block=True, timeout_ms=1000)
    r = cache.get_async(0, torch.device("cuda"))
    kg, vg, ev = r
    torch.cuda.current_stream().wait_event(ev)
    k, v, L, _ = cache.get_snapshot(0)
    assert torch.equal(kg.cpu(), k) and torch.equal(vg.cpu(), v) and L == 20
    cache.mark_layer_buffer_consumed(0, torch.cuda.current_stream())
    assert cache.get_async(1, torch.device("cuda")) is None
    assert cache.get_sparse_async_uva(1, torch.device("cuda"), torch.tensor([0])) is None
    cache.shutdown()
    with pytest.raises(RuntimeError):
        cache.submit_append(0, kn, kn)


def test_engine_paged_append_and_writeback(built_lib):
    """OffloadKV.append: K rows land in their HBM pages, K and V rows in the host store."""
    from mserve_b200.engine import OffloadKV
    g = torch.Generator().manual_seed(2)
    B, Hq, Hkv, D, C = 3, 8, 2, 128, 200
    eng = OffloadKV(2, B, Hq, Hkv, D, C, top_k=16, recent=4)
    ok = [[None, None] for _ in range(B)]
    for n_new in ([37, 5, 0], [1, 1, 1], [16, 40, 99]):
        n = max(n_new)
        eng.reserve(n_new)
        kl, vl = [], []
        for layer in range(2):
            kn = torch.randn(B, Hkv, n, D, generator=g).to(torch.bfloat16)
            vn = torch.randn(B, Hkv, n, D, generator=g).to(torch.bfloat16)
            eng.append_layer(layer, kn.cuda(), vn.cuda())
            kl.append(kn), vl.append(vn)
        eng.commit()
        torch.cuda.synchronize()
        for b in range(B):
            kb = to_numpy_bits(kl[1][b:b + 1, :, :n_new[b]])
            vb = to_numpy_bits(vl[1][b:b + 1, :, :n_new[b]])
            ok[b] = list(ko.cat_truncate(ok[b][0], ok[b][1], kb, vb, C))
    ops_status = __import__("mserve_b200.ops", fromlist=["check_status"])
    ops_status.check_status(torch.device("cuda"))
    pt = eng.page_table.cpu().numpy()
    pool = to_numpy_bits(eng.pool_k[1])
    for b in range(B):
        hk, hv = eng.host_logical(1, b)
        np.testing.assert_array_equal(to_numpy_bits(hk), ok[b][0][0])
        np.testing.assert_array_equal(to_numpy_bits(hv), ok[b][1][0])
        L = int(eng.len_h[b])
        pages = np.stack([pool[pt[b, t // 16], :, t % 16] for t in range(L)], axis=1)
        np.testing.assert_array_equal(pages, ok[b][0][0])


def test_page_writeback_to_host(built_lib):
    """Pages -> host rows (the write-back of evicted pages), ring-aware, against the oracle."""
    from mserve_b200 import ops
    g = torch.Generator().manual_seed(8)
    B, H, D, ps, maxp, C = 2, 4, 128, 16, 6, 64
    P = B * maxp
    pool_k = torch.randn(P, H, ps, D, generator=g).to(torch.bfloat16)
    pool_v = torch.randn(P, H, ps, D, generator=g).to(torch.bfloat16)
    pt = torch.randperm(P, generator=g).to(torch.int32).view(B, maxp)
    host_k = ops.host_empty((B, H, C, D), torch.bfloat16)
    host_v = ops.host_empty((B, H, C, D), torch.bfloat16)
    host_k.zero_(), host_v.zero_()
    tok_start = torch.tensor([16, 5], dtype=torch.int32)
    counts = torch.tensor([32, 50], dtype=torch.int32)
    ring = torch.tensor([0, 40], dtype=torch.int32)
    dev = torch.device("cuda")
    src = ops.paged_rows(pool_k.to(dev), pool_v.to(dev), pt.to(dev), len_scalar=maxp * ps, tok0=tok_start.to(dev))
    dst = ops.strided_rows(host_k, host_v, len_scalar=C, ring_start=ring.to(dev), ring_cap=C,
                           tok0=tok_start.to(dev), device=dev)
    ops.copy_rows(src, dst, batch=B, num_tokens=50, counts=counts.to(dev), device=dev)
    torch.cuda.synchronize()
    ops.check_status(dev)
    ek = np.zeros((B, H, C, D), dtype=np.int16)
    ev = np.zeros_like(ek)
    ko.page_writeback(to_numpy_bits(pool_k), to_numpy_bits(pool_v), pt.numpy(), ek, ev, tok_start.numpy(),
                      counts.numpy(), ring_start=ring.numpy(), ring_cap=C)
    np.testing.assert_array_equal(to_numpy_bits(host_k), ek)
    np.testing.assert_array_equal(to_numpy_bits(host_v), ev)


def test_get_sparse_async_matches_reference_golden(built_lib, golden):
    """get_sparse_async (kv_cache.py:545-629): the rows land in the cache's reusable per-layer
    device buffers, copied on its own stream, and equal the reference's own get_sparse_async
    output on the golden cache; later calls with more and fewer indices reuse (and grow) the
    buffers and stay bit-exact with the oracle."""
    from mserve_b200.kv_cache import CPUKVCache
    k = from_bits(golden["sparse/k"], torch.bfloat16)
    v = from_bits(golden["sparse/v"], torch.bfloat16)
    B, H, T, D = k.shape
    cache = CPUKVCache(num_layers=2, max_len=T + 16)
    assert cache.submit_append(1, k.cuda(), v.cuda())
    idx = torch.from_numpy(golden["sparse/idx"])
    ks, vs, ev = cache.get_sparse_async(1, torch.device("cuda"), idx)
    assert ks.shape == (B, H, idx.numel(), D)
    torch.cuda.current_stream().wait_event(ev)
    np.testing.assert_array_equal(to_numpy_bits(ks), golden["sparse/k_sel"].view(np.int16))
    np.testing.assert_array_equal(to_numpy_bits(vs), golden["sparse/v_sel"].view(np.int16))
    kb = to_numpy_bits(k)
    vb = to_numpy_bits(v)
    g = torch.Generator().manual_seed(5)
    storages = []
    for S, on_gpu in ((3 * idx.numel(), False), (7, True), (idx.numel() + 1, False)):
        sel = torch.randint(0, T, (S,), generator=g)
        ks2, vs2, ev2 = cache.get_sparse_async(1, torch.device("cuda"), sel.cuda() if on_gpu else sel)
        torch.cuda.current_stream().wait_event(ev2)
        ek, evv = ko.index_select_gather(kb, vb, sel.numpy())
        np.testing.assert_array_equal(to_numpy_bits(ks2), ek)
        np.testing.assert_array_equal(to_numpy_bits(vs2), evv)
        storages.append(ks2.untyped_storage().data_ptr())
    # once grown to the largest selection, later calls of the layer reuse the same buffer
    assert storages[0] == storages[1] == storages[2]
    assert ks2.untyped_storage().nbytes() >= B * H * 3 * idx.numel() * D * 2
    with pytest.raises(RuntimeError, match="out of range"):
        cache.get_sparse_async(1, torch.device("cuda"), torch.tensor([T]))
    assert cache.get_sparse_async(0, torch.device("cuda"), idx) is None
    cache.shutdown()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32, torch.float8_e4m3fn])
def test_get_full_kv_matches_oracle(built_lib, dtype):
    """get_full_kv (kv_cache.py:631-643) on CUDA tensors runs the row-copy kernel: bit-exact with
    the oracle's concatenation for contiguous and strided past/new tensors and empty parts."""
    from mserve_b200.kv_cache import CPUKVCache
    g = torch.Generator().manual_seed(11)

    def rnd(*shape):
        return (torch.randn(*shape, generator=g) * 3).to(dtype).cuda()
    B, H, T, n, D = 2, 4, 300, 5, 128
    cases = [
        ((rnd(B, H, T, D), rnd(B, H, T, D)), rnd(B, H, n, D), rnd(B, H, n, D)),
        # strided views: a token slice of a larger cache, and a [B, T, H, D] tensor seen as [B, H, T, D]
        ((rnd(B, H, T + 40, D)[:, :, 17:17 + T], rnd(B, T, H, D).transpose(1, 2)), rnd(B, H, n, D),
         rnd(B, n, H, D).transpose(1, 2)),
        ((rnd(B, H, 0, D), rnd(B, H, 0, D)), rnd(B, H, 1, D), rnd(B, H, 1, D)),
        ((rnd(B, H, T, D), rnd(B, H, T, D)), rnd(B, H, 0, D), rnd(B, H, 0, D)),
    ]
    for past, kn, vn in cases:
        k, v = CPUKVCache.get_full_kv(past, kn, vn)
        torch.cuda.synchronize()
        ek, ev = ko.full_kv((to_numpy_bits(past[0]), to_numpy_bits(past[1])), to_numpy_bits(kn), to_numpy_bits(vn))
        assert k.is_cuda and k.is_contiguous() and k.dtype == dtype
        np.testing.assert_array_equal(to_numpy_bits(k), ek)
        np.testing.assert_array_equal(to_numpy_bits(v), ev)
    k, v = CPUKVCache.get_full_kv(None, kn, vn)
    assert k is kn and v is vn
    with pytest.raises(RuntimeError, match="Sizes of tensors must match"):
        CPUKVCache.get_full_kv((rnd(B, H, T, D), rnd(B, H, T, D)), rnd(B, H + 1, n, D), rnd(B, H + 1, n, D))
