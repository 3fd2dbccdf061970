"""The larger decode-selection shapes, one layer each, through the engine, against the oracle.

* Qwen2.5-VL-32B shape: 16 sequences x 32768 tokens, 40 query / 8 KV heads, head_dim 128,
  bf16, KV ~N(0,1) (seed 2), top-4096 plus the last 256 tokens per (sequence, KV head).
* LLaVA-v1.6-34B multi-turn shape (4 of its 32 sequences; every per-sequence size as in the
  full batch): 56 query / 8 KV heads, context lengths uniform in [4096, 65536] (seed 3); a
  turn appends 2880 image tokens (5 tiles x 576) and 64 text tokens into 16-token HBM key
  pages with the rows written through to the pinned host store; then decode selects the
  top ceil(10% of L_b) tokens per (sequence, KV head).

Checks: scores within 1e-3 of the fp64 oracle; index sets exactly the oracle's ranking of
the GPU's fp32 scores; host store, key pages and gathered rows bit-exact; attention within
2e-2 (bf16).
"""
import math

import numpy as np
import pytest
import torch

from conftest import to_numpy_bits
from test_select_gpu import scores_close_error
from oracle import kv_oracle as ko

pytestmark = pytest.mark.gpu


def _check_layer(eng, layer, q, ks, vs, lens, top_k, recent):
    """ks/vs: per-sequence bf16 CPU tensors [Hkv, L_b, D] (the logical cache)."""
    B, Hkv, D = eng.B, eng.Hkv, eng.D
    out = eng.decode_layer(layer, q.cuda())
    torch.cuda.synchronize()
    bufs = eng.buffers()
    scores = bufs.scores.cpu().numpy()
    idx, cnt = bufs.idx.cpu().numpy(), bufs.counts.cpu().numpy()
    qn = q.float().numpy()
    # 1. scores (per sequence, fp64 oracle)
    for b in range(B):
        L = lens[b]
        ref = ko.gqa_scores(qn[b:b + 1], ks[b].float().numpy()[None])[0]
        s = scores[b, :, :L].astype(np.float64)
        assert scores_close_error(s, ref) < 1e-3, f"scores of sequence {b}"
    # 2. selection: the oracle's rule on the GPU's fp32 scores
    sel, rcnt = ko.select_topk_window(scores.reshape(B * Hkv, -1), top_k=top_k, recent=recent,
                                      lens=np.asarray(lens), sel_per_batch=Hkv)
    np.testing.assert_array_equal(cnt, rcnt)
    for j in range(B * Hkv):
        np.testing.assert_array_equal(idx[j, :cnt[j]], sel[j])
    # 3. gathered rows bit-exact; 4. attention
    kb, vb = to_numpy_bits(bufs.k_sel), to_numpy_bits(bufs.v_sel)
    S = bufs.k_sel.shape[2]
    o = out.float().cpu().numpy()
    for b in range(B):
        k_sel = np.zeros((1, Hkv, S, D))
        v_sel = np.zeros_like(k_sel)
        kbits, vbits = ks[b].view(torch.int16).numpy(), vs[b].view(torch.int16).numpy()
        kn, vn = ks[b].float().numpy(), vs[b].float().numpy()
        for h in range(Hkv):
            j = b * Hkv + h
            np.testing.assert_array_equal(kb[b, h, :cnt[j]], kbits[h, sel[j]])
            np.testing.assert_array_equal(vb[b, h, :cnt[j]], vbits[h, sel[j]])
            k_sel[0, h, :cnt[j]] = kn[h, sel[j]]
            v_sel[0, h, :cnt[j]] = vn[h, sel[j]]
        ref = ko.sparse_sdpa_attention(q[b:b + 1].double().numpy()[:, :, None, :], k_sel, v_sel,
                                       counts=cnt[b * Hkv:(b + 1) * Hkv].reshape(1, Hkv))
        assert np.abs(o[b:b + 1] - ref).max() / np.abs(ref).max() < 2e-2, f"attention of sequence {b}"
    from mserve_b200 import ops
    ops.check_status(torch.device("cuda"))


def test_qwen32b_shape_layer(built_lib):
    from mserve_b200.engine import OffloadKV
    B, Hq, Hkv, D, T, K, R = 16, 40, 8, 128, 32768, 4096, 256
    g = torch.Generator().manual_seed(2)
    eng = OffloadKV(1, B, Hq, Hkv, D, T, top_k=K, recent=R)
    eng.reserve([T] * B)
    k_dev = torch.empty(B, Hkv, T, D, dtype=torch.bfloat16, device="cuda")
    v_dev = torch.empty_like(k_dev)
    ks, vs = [], []
    for b in range(B):
        k = torch.randn(Hkv, T, D, generator=g).to(torch.bfloat16)
        v = torch.randn(Hkv, T, D, generator=g).to(torch.bfloat16)
        k_dev[b].copy_(k)
        v_dev[b].copy_(v)
        ks.append(k), vs.append(v)
    eng.append_layer(0, k_dev, v_dev)
    eng.commit()
    del k_dev, v_dev
    q = torch.randn(B, Hq, D, generator=g).to(torch.bfloat16)
    _check_layer(eng, 0, q, ks, vs, [T] * B, K, R)


def test_llava34b_multiturn_shape(built_lib):
    from mserve_b200.engine import OffloadKV
    B, Hq, Hkv, D, ps = 4, 56, 8, 128, 16
    n_img, n_txt = 5 * 576, 64
    rng = np.random.default_rng(3)
    ctx = [int(x) for x in rng.integers(4096, 65536, size=32, endpoint=True)[:B]]
    cap = max(ctx) + n_img + n_txt
    eng = OffloadKV(1, B, Hq, Hkv, D, cap, top_k_ratio=0.1, recent=0, page_size=ps)
    g = torch.Generator().manual_seed(3)
    parts_k, parts_v = [[] for _ in range(B)], [[] for _ in range(B)]

    def turn(n_new, text_from):
        """Appends n_new[b] tokens per sequence; tokens >= text_from[b] of the turn are text."""
        n_max = max(n_new)
        k_new = torch.zeros(B, Hkv, n_max, D, dtype=torch.bfloat16)
        v_new = torch.zeros_like(k_new)
        for b in range(B):
            k = torch.randn(Hkv, n_new[b], D, generator=g)
            v = torch.randn(Hkv, n_new[b], D, generator=g)
            k[:, text_from[b]:] *= 0.5
            v[:, text_from[b]:] *= 0.5
            k_new[b, :, :n_new[b]] = k.to(torch.bfloat16)
            v_new[b, :, :n_new[b]] = v.to(torch.bfloat16)
            parts_k[b].append(k_new[b, :, :n_new[b]])
            parts_v[b].append(v_new[b, :, :n_new[b]])
        eng.reserve(n_new)
        eng.append_layer(0, k_new.cuda(), v_new.cuda())
        eng.commit()

    turn(ctx, [c for c in ctx])                         # the existing context
    turn([n_img + n_txt] * B, [n_img] * B)              # one turn: 2880 image + 64 text tokens
    lens = [c + n_img + n_txt for c in ctx]
    assert list(eng.len_h) == lens
    assert list(eng.topk_h) == [math.ceil(0.1 * L) for L in lens]
    kl = [torch.cat(p, dim=1) for p in parts_k]
    vl = [torch.cat(p, dim=1) for p in parts_v]
    # host store (ring order) and HBM key pages hold exactly the appended rows
    pool = to_numpy_bits(eng.pool_k[0])
    pt = eng.page_table.cpu().numpy()
    for b in range(B):
        hk, hv = eng.host_logical(0, b)
        assert torch.equal(hk.view(torch.int16), kl[b].view(torch.int16))
        assert torch.equal(hv.view(torch.int16), vl[b].view(torch.int16))
        L = lens[b]
        pages = pool[pt[b, :(L + ps - 1) // ps]]                 # [n_pages, Hkv, ps, D]
        paged = pages.transpose(1, 0, 2, 3).reshape(Hkv, -1, D)[:, :L]
        np.testing.assert_array_equal(paged, to_numpy_bits(kl[b]))
    q = torch.randn(B, Hq, D, generator=g).to(torch.bfloat16)
    _check_layer(eng, 0, q, kl, vl, lens, [int(x) for x in eng.topk_h], 0)


def test_ratio_selection_pipelined_graph(built_lib):
    """Per-sequence k (top_k_ratio) through the chunked three-stream step and its CUDA graph:
    bit-identical to layer-by-layer decoding."""
    from mserve_b200.engine import OffloadKV
    B, Hq, Hkv, D, L = 5, 56, 8, 128, 2
    lens = [900, 4000, 77, 2500, 1600]
    eng = OffloadKV(L, B, Hq, Hkv, D, 4096, top_k_ratio=0.1, recent=16)
    g = torch.Generator().manual_seed(11)
    eng.reserve(lens)
    for layer in range(L):
        k = torch.randn(B, Hkv, max(lens), D, generator=g).to(torch.bfloat16)
        v = torch.randn(B, Hkv, max(lens), D, generator=g).to(torch.bfloat16)
        eng.append_layer(layer, k.cuda(), v.cuda())
    eng.commit()
    q = torch.randn(L, B, Hq, D, generator=g).to(torch.bfloat16).cuda()
    ref = torch.stack([eng.decode_layer(layer, q[layer]).clone() for layer in range(L)])
    cnt = eng.buffers().counts.view(B, Hkv).cpu()
    for b in range(B):
        expect = min(math.ceil(0.1 * lens[b]), max(lens[b] - 16, 0)) + min(16, lens[b])
        assert (cnt[b] == expect).all()
    out = torch.zeros(L, B, Hq, 1, D, dtype=torch.bfloat16, device="cuda")
    graph = eng.capture_decode_step(q, out, chunks=3)
    out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
