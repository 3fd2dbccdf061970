"""The oracle pinned against the reference's own outputs (tests/golden/reference_vectors.npz,
produced by tests/golden/make_golden.py from MServe's Python functions run on CPU), and the C
restatement (oracle/oracle_kv.c) pinned against the numpy oracle.  CPU only."""
import numpy as np
import pytest

from oracle import kv_oracle as ko

CTI = ["cti_f64_score", "cti_f64_norm", "cti_f64_q3", "cti_f64_short", "cti_f64_b2", "cti_f32_score",
       "cti_bf16_score"]


def _arr(golden, key, dt):
    a = golden[key]
    return ko.bf16_to_f32(a) if "bfloat16" in dt else a


@pytest.mark.parametrize("case", CTI)
def test_compute_token_importance_matches_reference(golden, case):
    B, Hq, Hkv, Q, T, D, method, mn = [int(x) for x in golden[f"{case}/meta"]]
    dt = str(golden[f"{case}/dtype"])
    ratio = float(golden[f"{case}/ratio"][0])
    q, k = _arr(golden, f"{case}/q", dt), _arr(golden, f"{case}/k", dt)
    mname = ["attention_score", "norm"][method]
    ref = golden[f"{case}/idx"]
    if "float64" in dt:
        got = ko.compute_token_importance(q, k, mname, ratio, mn)
        np.testing.assert_array_equal(got, ref)       # exact in fp64
        return
    # fp32 / bf16: the reference ranked scores computed in that precision; the sets agree
    # except for tokens whose fp64 score is within the precision of the threshold.
    got = ko.compute_token_importance(q, k, mname, ratio, mn).reshape(B, -1)
    per = ko.gqa_scores(q[:, :, -1].astype(np.float64), k.astype(np.float64), method=mname)
    scores = per.sum(axis=1)
    rtol = 2e-2 if "bfloat16" in dt else 1e-5
    for b in range(B):
        diff = set(got[b].tolist()) ^ set(ref.reshape(B, -1)[b].tolist())
        kth = np.sort(scores[b])[::-1][got.shape[1] - 1]
        tol = rtol * np.abs(scores[b]).max()
        assert all(abs(scores[b, t] - kth) <= tol for t in diff)


def test_repeat_kv_matches_reference(golden):
    np.testing.assert_array_equal(ko.repeat_kv(golden["repeat_kv/x"], 4), golden["repeat_kv/out"])


@pytest.mark.parametrize("case", ["attn_f64", "attn_bf16", "attn_f32_q2"])
def test_sparse_attention_matches_reference(golden, case):
    dt = str(golden[f"{case}/dtype"])
    q, k, v = (_arr(golden, f"{case}/{n}", dt) for n in ("q", "k_sel", "v_sel"))
    ref = _arr(golden, f"{case}/out", dt)
    got = ko.sparse_sdpa_attention(q, k, v)
    rtol = 1e-12 if "float64" in dt else (1e-5 if "float32" in dt else 2e-2)
    assert np.abs(got - ref).max() <= rtol * np.abs(ref).max()


def test_append_cat_truncate_matches_reference(golden):
    """CPUKVCache.append_new (cat, keep last max_len) -- bit-exact, and the ring form too."""
    max_len = int(golden["append/max_len"])
    ok = ov = None
    ring = None
    for i in range(7):
        kn, vn = golden[f"append/step{i}/k_new"], golden[f"append/step{i}/v_new"]
        ok, ov = ko.cat_truncate(ok, ov, kn, vn, max_len)
        np.testing.assert_array_equal(ok, golden[f"append/step{i}/k"])
        np.testing.assert_array_equal(ov, golden[f"append/step{i}/v"])
        assert ok.shape[2] == int(golden[f"append/step{i}/meta"][0])
        if ring is None:
            ring = ko.RingStore(kn.shape[0], kn.shape[1], max_len, kn.shape[3:], kn.dtype)
        ring.append(kn, vn)
        rk, rv = ring.logical(0)
        np.testing.assert_array_equal(rk, golden[f"append/step{i}/k"][0])
        np.testing.assert_array_equal(rv, golden[f"append/step{i}/v"][0])


def test_gather_matches_reference_get_sparse_async(golden):
    k, v, idx = golden["sparse/k"], golden["sparse/v"], golden["sparse/idx"]
    gk, gv = ko.index_select_gather(k, v, idx)
    np.testing.assert_array_equal(gk, golden["sparse/k_sel"])
    np.testing.assert_array_equal(gv, golden["sparse/v_sel"])
    gk2, gv2, mask, oob = ko.gather_segments(k, v, idx)
    assert not oob and mask.all()
    np.testing.assert_array_equal(gk2, gk)


def test_bf16_roundtrip():
    x = np.random.default_rng(0).standard_normal(1000).astype(np.float32)
    b = ko.f32_to_bf16(x)
    y = ko.bf16_to_f32(b)
    assert np.abs(y - x).max() <= np.abs(x).max() * 2 ** -8
    np.testing.assert_array_equal(ko.f32_to_bf16(y), b)


def test_select_rule_edge_cases():
    rows = np.array([[1, 3, 3, 2, 3, 0]], dtype=np.float32)
    sel, cnt = ko.select_topk_window(rows, top_k=2, recent=0)
    np.testing.assert_array_equal(sel[0], [1, 2])           # ties: lower index first
    sel, cnt = ko.select_topk_window(rows, top_k=2, recent=2)
    np.testing.assert_array_equal(sel[0], [1, 2, 4, 5])     # window [4, 6) appended
    sel, cnt = ko.select_topk_window(rows, top_k=9, recent=10)
    np.testing.assert_array_equal(sel[0], np.arange(6))     # L < R: the window is everything
    rows = np.array([[np.nan, -1, 5, -0.0, 0.0]], dtype=np.float32)
    sel, _ = ko.select_topk_window(rows, top_k=3, recent=0)
    np.testing.assert_array_equal(sel[0], [0, 2, 4])        # NaN highest, +0 above -0
