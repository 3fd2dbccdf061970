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
