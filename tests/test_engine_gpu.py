"""End-to-end decode layer of the offload engine against the oracle.

score (HBM key pages) -> top-k ∪ window per (sequence, KV head) -> gather from the host
store -> attention.  The selection is checked exactly by ranking the GPU's own fp32 scores
with the oracle's rule; gathered rows bit-exactly; the output within 2e-2 (bf16).
"""
import numpy as np
import pytest
import torch

from conftest import to_numpy_bits
from oracle import kv_oracle as ko

pytestmark = pytest.mark.gpu


def _build(B, Hq, Hkv, D, T, K, R, layers=2, seed=0, lens=None):
    from mserve_b200.engine import OffloadKV
    g = torch.Generator().manual_seed(seed)
    eng = OffloadKV(layers, B, Hq, Hkv, D, T + 32, top_k=K, recent=R)
    lens = lens or [T] * B
    eng.reserve(lens)
    ks, vs = [], []
    for layer in range(layers):
        k = torch.randn(B, Hkv, T, D, generator=g).to(torch.bfloat16)
        v = torch.randn(B, Hkv, T, D, generator=g).to(torch.bfloat16)
        eng.append_layer(layer, k.cuda(), v.cuda())
        ks.append(k), vs.append(v)
    eng.commit()
    return eng, ks, vs, g


@pytest.mark.parametrize("B,Hq,Hkv,T,K,R,lens", [(8, 28, 4, 2048, 256, 32, None), (2, 8, 2, 700, 100, 0, [700, 333]),
                                                 (3, 28, 4, 500, 600, 16, [500, 20, 499])])
def test_decode_layer_matches_oracle(built_lib, B, Hq, Hkv, T, K, R, lens):
    D = 128
    eng, ks, vs, g = _build(B, Hq, Hkv, D, T, K, R, lens=lens)
    lens = lens or [T] * B
    q = torch.randn(B, Hq, D, generator=g).to(torch.bfloat16)
    layer = 1
    out = eng.decode_layer(layer, q.cuda())
    torch.cuda.synchronize()
    bufs = eng.buffers()
    scores = bufs.scores.cpu().numpy()
    idx = bufs.idx.cpu().numpy()
    cnt = bufs.counts.cpu().numpy()
    kn, vn = ks[layer].float().numpy(), vs[layer].float().numpy()
    # 1. scores within 1e-3 of the fp64 oracle
    ref_scores = ko.gqa_scores(q.float().numpy(), kn, lens=np.asarray(lens))
    for b in range(B):
        L = lens[b]
        s, r = scores[b, :, :L].astype(np.float64), ref_scores[b, :, :L]
        assert (np.abs(s - r) / (np.abs(r) + np.abs(r).mean())).max() < 1e-3
    # 2. selection: exactly the oracle's rule applied to the GPU's fp32 scores
    sel, rcnt = ko.select_topk_window(scores.reshape(B * Hkv, -1), top_k=K, recent=R,
                                      lens=np.asarray(lens), sel_per_batch=Hkv)
    np.testing.assert_array_equal(cnt, rcnt)
    for j in range(B * Hkv):
        np.testing.assert_array_equal(idx[j, :cnt[j]], sel[j])
    # 3. gathered rows bit-exact
    kb, vb = to_numpy_bits(bufs.k_sel), to_numpy_bits(bufs.v_sel)
    hk, hv = to_numpy_bits(ks[layer]), to_numpy_bits(vs[layer])
    for j in range(B * Hkv):
        b, h = divmod(j, Hkv)
        np.testing.assert_array_equal(kb[b, h, :cnt[j]], hk[b, h, sel[j]])
        np.testing.assert_array_equal(vb[b, h, :cnt[j]], hv[b, h, sel[j]])
    # 4. attention over the selection
    k_sel = np.zeros((B, Hkv, bufs.k_sel.shape[2], D))
    v_sel = np.zeros_like(k_sel)
    for j in range(B * Hkv):
        b, h = divmod(j, Hkv)
        k_sel[b, h, :cnt[j]] = kn[b, h, sel[j]]
        v_sel[b, h, :cnt[j]] = vn[b, h, sel[j]]
    ref = ko.sparse_sdpa_attention(q.double().numpy()[:, :, None, :], k_sel, v_sel, counts=cnt.reshape(B, Hkv))
    o = out.float().cpu().numpy()
    assert np.abs(o - ref).max() / np.abs(ref).max() < 2e-2
    from mserve_b200 import ops
    ops.check_status(torch.device("cuda"))


@pytest.mark.parametrize("chunks", [1, 3, 4])
def test_pipelined_step_and_graph_match_per_layer(built_lib, chunks):
    """decode_step (chunked, three streams) and its CUDA graph give bit-identical outputs to
    running decode_layer layer by layer."""
    B, Hq, Hkv, D, T, K, R, L = 6, 28, 4, 128, 1500, 200, 16, 3
    eng, ks, vs, g = _build(B, Hq, Hkv, D, T, K, R, layers=L, seed=7)
    q = torch.randn(L, B, Hq, D, generator=g).to(torch.bfloat16).cuda()
    ref = torch.stack([eng.decode_layer(layer, q[layer]).clone() for layer in range(L)])
    out = torch.zeros(L, B, Hq, 1, D, dtype=torch.bfloat16, device="cuda")
    eng.decode_step(q, out, chunks=chunks)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    out.zero_()
    graph = eng.capture_decode_step(q, out, chunks=chunks)
    out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    from mserve_b200 import ops
    ops.check_status(torch.device("cuda"))


@pytest.mark.parametrize("dtype,D", [(torch.float16, 128), (torch.bfloat16, 64), (torch.float16, 64)])
def test_decode_layer_dtypes_and_head_dims(built_lib, dtype, D):
    """The whole decode layer with fp16 keys/values and with head_dim 64 (the 16-bit streaming
    score path and the tensor-core attention path at both sizes) against the oracle."""
    from mserve_b200.engine import OffloadKV
    B, Hq, Hkv, T, K, R = 3, 16, 4, 3000, 300, 32
    g = torch.Generator().manual_seed(D + (1 if dtype == torch.float16 else 0))
    eng = OffloadKV(1, B, Hq, Hkv, D, T + 16, top_k=K, recent=R, dtype=dtype)
    lens = [3000, 2047, 1000]
    eng.reserve(lens)
    k = torch.randn(B, Hkv, T, D, generator=g).to(dtype)
    v = torch.randn(B, Hkv, T, D, generator=g).to(dtype)
    eng.append_layer(0, k.cuda(), v.cuda())
    eng.commit()
    q = torch.randn(B, Hq, D, generator=g).to(dtype)
    out = eng.decode_layer(0, q.cuda())
    torch.cuda.synchronize()
    bufs = eng.buffers()
    scores, idx, cnt = bufs.scores.cpu().numpy(), bufs.idx.cpu().numpy(), bufs.counts.cpu().numpy()
    kn, vn = k.float().numpy(), v.float().numpy()
    ref_scores = ko.gqa_scores(q.float().numpy(), kn, lens=np.asarray(lens))
    for b in range(B):
        L = lens[b]
        s, r = scores[b, :, :L].astype(np.float64), ref_scores[b, :, :L]
        assert (np.abs(s - r) / (np.abs(r) + np.abs(r).mean())).max() < 1e-3
    sel, rcnt = ko.select_topk_window(scores.reshape(B * Hkv, -1), top_k=K, recent=R, lens=np.asarray(lens),
                                      sel_per_batch=Hkv)
    np.testing.assert_array_equal(cnt, rcnt)
    kb, hk = to_numpy_bits(bufs.k_sel), to_numpy_bits(k)
    k_sel = np.zeros((B, Hkv, bufs.k_sel.shape[2], D))
    v_sel = np.zeros_like(k_sel)
    for j in range(B * Hkv):
        b, h = divmod(j, Hkv)
        np.testing.assert_array_equal(idx[j, :cnt[j]], sel[j])
        np.testing.assert_array_equal(kb[b, h, :cnt[j]], hk[b, h, sel[j]])
        k_sel[b, h, :cnt[j]] = kn[b, h, sel[j]]
        v_sel[b, h, :cnt[j]] = vn[b, h, sel[j]]
    ref = ko.sparse_sdpa_attention(q.double().numpy()[:, :, None, :], k_sel, v_sel, counts=cnt.reshape(B, Hkv))
    o = out.float().cpu().numpy()
    assert np.abs(o - ref).max() / np.abs(ref).max() < 2e-2


def _twin_engines(B, Hq, Hkv, D, lens, C, L, seed, **sel):
    """Two engines holding the same prefilled cache (lengths `lens`)."""
    from mserve_b200.engine import OffloadKV
    engs = [OffloadKV(L, B, Hq, Hkv, D, C, **sel) for _ in range(2)]
    g = torch.Generator().manual_seed(seed)
    T = max(lens)
    rows = [(torch.randn(B, Hkv, T, D, generator=g).to(torch.bfloat16).cuda(),
             torch.randn(B, Hkv, T, D, generator=g).to(torch.bfloat16).cuda()) for _ in range(L)]
    for eng in engs:
        eng.reserve(lens)
        for layer, (k, v) in enumerate(rows):
            eng.append_layer(layer, k, v)
        eng.commit()
    return engs, g


@pytest.mark.parametrize("sel", [dict(top_k=64, recent=8), dict(top_k_ratio=0.125, recent=4), dict(top_k=40)])
def test_decode_loop_appends_its_token_in_the_graph(built_lib, sel):
    """A decode loop whose step writes its own token: begin_step() then one CUDA graph captured
    once with a length bound, replayed every step while the cache grows across page
    boundaries, against the same steps done eagerly (reserve / append_layer / commit, then
    decode_layer per layer): outputs bit-identical every step; host store and HBM key pages
    bit-identical at the end."""
    B, Hq, Hkv, D, L, steps = 5, 16, 4, 128, 3, 21
    lens = [300, 31, 47, 16, 129]
    C = max(lens) + steps + 8
    (eng, ref), g = _twin_engines(B, Hq, Hkv, D, lens, C, L, seed=11, **sel)
    dev = torch.device("cuda")
    q = torch.zeros(L, B, Hq, D, dtype=torch.bfloat16, device=dev)
    kn = torch.zeros(L, B, Hkv, D, dtype=torch.bfloat16, device=dev)
    vn = torch.zeros_like(kn)
    out = torch.zeros(L, B, Hq, 1, D, dtype=torch.bfloat16, device=dev)
    graph = None
    for step in range(steps):
        q.copy_(torch.randn(L, B, Hq, D, generator=g).to(torch.bfloat16))
        kn.copy_(torch.randn(L, B, Hkv, D, generator=g).to(torch.bfloat16))
        vn.copy_(torch.randn(L, B, Hkv, D, generator=g).to(torch.bfloat16))
        eng.begin_step()
        if graph is None:          # the capture runs this step once
            graph = eng.capture_decode_step(q, out, chunks=3, k_new=kn, v_new=vn, t_bound=C)
        else:
            graph.replay()
        ref.reserve([1] * B)
        for layer in range(L):
            ref.append_layer(layer, kn[layer].unsqueeze(2), vn[layer].unsqueeze(2))
        ref.commit()
        want = torch.stack([ref.decode_layer(layer, q[layer]).clone() for layer in range(L)])
        torch.cuda.synchronize()
        assert torch.equal(out, want), f"step {step}"
    assert (eng.len_h == ref.len_h).all() and (eng.len_h == np.asarray(lens) + steps).all()
    assert torch.equal(eng.lens, ref.lens) and torch.equal(eng.split, ref.split)
    pt = eng.page_table.cpu().numpy()
    pt_ref = ref.page_table.cpu().numpy()
    for layer in range(L):
        for b in range(B):
            hk, hv = eng.host_logical(layer, b)
            rk, rv = ref.host_logical(layer, b)
            assert torch.equal(hk, rk) and torch.equal(hv, rv)
            n = int(eng.len_h[b])
            pool, pool_ref = to_numpy_bits(eng.pool_k[layer]), to_numpy_bits(ref.pool_k[layer])
            mine = np.stack([pool[pt[b, t // 16], :, t % 16] for t in range(n)], axis=1)
            theirs = np.stack([pool_ref[pt_ref[b, t // 16], :, t % 16] for t in range(n)], axis=1)
            np.testing.assert_array_equal(mine, theirs)
    from mserve_b200 import ops
    ops.check_status(dev)


def test_begin_step_guards(built_lib):
    from mserve_b200.engine import OffloadKV
    eng = OffloadKV(1, 2, 4, 2, 64, 20, top_k=4, recent=2)
    eng.reserve([20, 3])
    k = torch.zeros(2, 2, 20, 64, dtype=torch.bfloat16, device="cuda")
    eng.append_layer(0, k, k)
    with pytest.raises(RuntimeError):
        eng.begin_step()                     # inside reserve()/commit()
    eng.commit()
    with pytest.raises(ValueError):
        eng.begin_step()                     # sequence 0 is full
    q = torch.zeros(1, 2, 4, 64, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(1, 2, 4, 1, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        eng.decode_step(q, out, k_new=torch.zeros(1, 2, 2, 64, dtype=torch.bfloat16, device="cuda"))
    with pytest.raises(ValueError):
        eng.decode_step(q, out, t_bound=21)
