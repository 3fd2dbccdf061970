"""The C restatement (oracle/oracle_kv.c, the timed CPU baseline) against the numpy oracle. CPU only."""
import ctypes as C
import math

import numpy as np
import pytest

from oracle import build_oracle
from oracle import kv_oracle as ko


@pytest.fixture(scope="module")
def clib():
    return build_oracle.load()


def _bf16(rng, shape, scale=1.0):
    return ko.f32_to_bf16(rng.standard_normal(shape).astype(np.float32) * scale)


def test_c_pipeline_matches_numpy_oracle(clib):
    rng = np.random.default_rng(0)
    B, Hq, Hkv, D, T, Cap, K, R = 2, 28, 4, 128, 900, 1000, 100, 16
    S = K + R
    hk, hv = _bf16(rng, (B, Hkv, Cap, D)), _bf16(rng, (B, Hkv, Cap, D))
    q = _bf16(rng, (B, Hq, D))
    nth = 4
    scores = np.empty((B * Hkv, T), dtype=np.float32)
    clib.okv_score_bf16(q.ctypes.data, hk.ctypes.data, Hkv * Cap * D, Cap * D, D, B, Hq, Hkv, T, D,
                        scores.ctypes.data, T, nth)
    ref = ko.gqa_scores(ko.bf16_to_f32(q), ko.bf16_to_f32(hk[:, :, :T]))
    assert np.abs(scores.reshape(B, Hkv, T) - ref).max() <= 1e-3 * (np.abs(ref).max())
    idx = np.empty((B * Hkv, S), dtype=np.int32)
    counts = np.empty(B * Hkv, dtype=np.int32)
    clib.okv_topk(scores.ctypes.data, T, B * Hkv, Hkv, None, T, K, R, idx.ctypes.data, S, counts.ctypes.data, nth)
    sel, rc = ko.select_topk_window(scores, top_k=K, recent=R, len_scalar=T)
    np.testing.assert_array_equal(counts, rc)
    for j in range(B * Hkv):
        np.testing.assert_array_equal(idx[j, :counts[j]], sel[j])
    ks = np.zeros((B, Hkv, S, D), dtype=np.uint16)
    vs = np.zeros_like(ks)
    clib.okv_gather(hk.ctypes.data, hv.ctypes.data, Hkv * Cap * D * 2, Cap * D * 2, D * 2, B, Hkv, idx.ctypes.data,
                    32, Hkv * S, S, S, counts.ctypes.data, ks.ctypes.data, vs.ctypes.data, D * 2, nth)
    ek, ev, mask, oob = ko.gather_segments(hk, hv, idx.reshape(B, Hkv, S), counts=counts.reshape(B, Hkv))
    assert not oob
    np.testing.assert_array_equal(ks, ek)
    np.testing.assert_array_equal(vs, ev)
    out = np.empty((B, Hq, D), dtype=np.float32)
    clib.okv_attention_bf16(q.ctypes.data, ks.ctypes.data, vs.ctypes.data, counts.ctypes.data, B, Hq, Hkv, S, D,
                            C.c_float(1.0 / math.sqrt(D)), out.ctypes.data, nth)
    ref = ko.sparse_sdpa_attention(ko.bf16_to_f32(q)[:, :, None, :], ko.bf16_to_f32(ks), ko.bf16_to_f32(vs),
                                   counts=counts.reshape(B, Hkv))[:, :, 0]
    assert np.abs(out - ref).max() <= 1e-4 * np.abs(ref).max()


def test_c_topk_ties_and_short(clib):
    rows = np.random.default_rng(1).integers(-2, 3, (5, 400)).astype(np.float32)
    rows[2, 7] = np.nan
    for K, R in [(50, 0), (399, 1), (0, 10), (500, 20)]:
        idx = np.empty((5, 1000), dtype=np.int32)
        cnt = np.empty(5, dtype=np.int32)
        clib.okv_topk(rows.ctypes.data, 400, 5, 1, None, 400, K, R, idx.ctypes.data, 1000, cnt.ctypes.data, 2)
        sel, rc = ko.select_topk_window(rows, top_k=K, recent=R)
        np.testing.assert_array_equal(cnt, rc)
        for j in range(5):
            np.testing.assert_array_equal(idx[j, :cnt[j]], sel[j])
