"""Parity of scoring (mskv_score) and selection (mskv_topk) with the oracle.

Scores: fp32 on the GPU vs fp64 in the oracle, within 1e-3 relative; only scores smaller than a
tenth of the mean magnitude (where a dot product cancels and its relative error means nothing)
are held to the absolute bound that 1e-3 gives at that size.  Selection: bit-exact index sets when the oracle ranks the GPU's own fp32 scores;
against the reference's golden outputs, index sets equal except at (near-)ties.
"""
import numpy as np
import pytest
import torch

from conftest import from_bits
from oracle import kv_oracle as ko

pytestmark = pytest.mark.gpu

SCORE_RTOL = 1e-3


def scores_close_error(got: np.ndarray, ref: np.ndarray) -> float:
    """max |got - ref| / max(|ref|, mean|ref| / 10): the relative error of every score except
    the near-zero ones, which are measured against a tenth of the mean magnitude."""
    floor = 0.1 * np.abs(ref).mean() + 1e-30
    return float((np.abs(got.astype(np.float64) - ref) / np.maximum(np.abs(ref), floor)).max())


def _assert_scores_close(got: np.ndarray, ref: np.ndarray):
    err = scores_close_error(got, ref)
    assert err <= SCORE_RTOL, f"max relative error {err:.3e}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("D", [64, 128, 256, 80])
@pytest.mark.parametrize("method", ["attention_score", "norm"])
def test_head_scores(built_lib, dtype, D, method):
    from mserve_b200.selection import head_scores
    g = torch.Generator().manual_seed(D)
    B, Hq, Hkv, T = 2, 28, 4, 1000
    q = torch.randn(B, Hq, D, generator=g).to(dtype)
    k = torch.randn(B, Hkv, T, D, generator=g).to(dtype)
    got = head_scores(q.cuda(), k.cuda(), method).cpu().numpy()
    ref = ko.gqa_scores(q.float().numpy(), k.float().numpy(), method=method)
    _assert_scores_close(got, ref)


def test_paged_scores_lens(built_lib):
    """Keys read through a page table, per-sequence lengths, pages scattered in the pool."""
    from mserve_b200 import ops
    g = torch.Generator().manual_seed(3)
    B, Hq, Hkv, D, ps, maxp = 3, 8, 2, 128, 16, 20
    P = B * maxp
    pool = torch.randn(P, Hkv, ps, D, generator=g).to(torch.bfloat16)
    perm = torch.randperm(P, generator=g).to(torch.int32).view(B, maxp)
    lens = torch.tensor([320, 17, 200], dtype=torch.int32)
    q = torch.randn(B, Hq, D, generator=g).to(torch.bfloat16)
    dev = torch.device("cuda")
    out = torch.full((B, Hkv, 320), float("nan"), device=dev)
    rows = ops.paged_rows(pool.to(dev), None, perm.to(dev), len_=lens.to(dev))
    ops.score(q.to(dev), rows, batch=B, kv_heads=Hkv, max_tokens=320, out=out)
    got = out.cpu().numpy()
    # logical K [B, Hkv, T, D] assembled on the CPU from the page table
    kl = pool.float().numpy()[perm.numpy()]             # [B, maxp, Hkv, ps, D]
    kl = kl.transpose(0, 2, 1, 3, 4).reshape(B, Hkv, maxp * ps, D)[:, :, :320]
    ref = ko.gqa_scores(q.float().numpy(), kl, lens=lens.numpy())
    for b in range(B):
        L = int(lens[b])
        _assert_scores_close(got[b, :, :L], ref[b, :, :L])
        assert np.isnan(got[b, :, L:]).all()            # beyond len: untouched


@pytest.mark.parametrize("T,K,R", [(16384, 2048, 128), (5000, 700, 0), (300, 300, 10), (300, 0, 16),
                                   (100, 50, 200), (1, 1, 1), (4096, 4095, 0)])
def test_topk_window_exact(built_lib, T, K, R):
    from mserve_b200 import ops
    g = torch.Generator().manual_seed(T + K)
    rows = torch.randn(6, T, generator=g)
    got, cnt = ops.topk(rows.cuda(), top_k=K, recent=R)
    ref, rcnt = ko.select_topk_window(rows.numpy(), top_k=K, recent=R)
    got, cnt = got.cpu().numpy(), cnt.cpu().numpy()
    np.testing.assert_array_equal(cnt, rcnt)
    for j in range(6):
        np.testing.assert_array_equal(got[j, :cnt[j]], ref[j])


def test_topk_ties_nan_lens_grouped(built_lib):
    """Heavy ties (quantised scores), NaN, -0.0/+0.0, per-sequence lengths and top_k,
    head-summed keys with a scale (the reference's mean over heads)."""
    from mserve_b200 import ops
    g = torch.Generator().manual_seed(9)
    B, Hk, T = 3, 4, 3000
    rows = torch.randint(-3, 4, (B * Hk, T), generator=g).float() * 0.5
    rows[0, 5] = float("nan")
    rows[1, :100] = -0.0
    lens = torch.tensor([3000, 1234, 77], dtype=torch.int32)
    topk_b = torch.tensor([500, 1000, 10], dtype=torch.int32)
    # per-head selections
    got, cnt = ops.topk(rows.cuda(), top_k=topk_b.cuda(), recent=32, len_=lens.cuda(), sel_per_batch=Hk)
    ref, rcnt = ko.select_topk_window(rows.numpy(), top_k=topk_b.numpy(), recent=32, lens=lens.numpy(),
                                      sel_per_batch=Hk)
    got, cnt = got.cpu().numpy(), cnt.cpu().numpy()
    np.testing.assert_array_equal(cnt, rcnt)
    for j in range(B * Hk):
        np.testing.assert_array_equal(got[j, :cnt[j]], ref[j])
    # one selection per sequence over the head-summed, scaled keys
    got, cnt = ops.topk(rows.cuda(), top_k=topk_b.cuda(), recent=0, len_=lens.cuda(), rows_per_sel=Hk,
                        sel_per_batch=1, scale=1.0 / 28)
    ref, rcnt = ko.select_topk_window(rows.numpy(), top_k=topk_b.numpy(), recent=0, lens=lens.numpy(),
                                      rows_per_sel=Hk, sel_per_batch=1, scale=1.0 / 28)
    got, cnt = got.cpu().numpy(), cnt.cpu().numpy()
    np.testing.assert_array_equal(cnt, rcnt)
    for j in range(B):
        np.testing.assert_array_equal(got[j, :cnt[j]], ref[j])


def _tie_tolerant_equal(got: np.ndarray, ref: np.ndarray, scores: np.ndarray, rtol: float):
    """Index sets equal except for tokens whose score is within rtol of the k-th score."""
    got_s, ref_s = set(got.tolist()), set(ref.tolist())
    assert len(got_s) == len(got) == len(ref)
    diff = got_s ^ ref_s
    if not diff:
        return
    kth = np.sort(scores)[::-1][len(ref) - 1]
    tol = rtol * (np.abs(scores).max() + 1e-30)
    bad = [t for t in diff if abs(scores[t] - kth) > tol]
    assert not bad, f"{len(bad)} indices differ away from the selection threshold"


@pytest.mark.parametrize("case", ["cti_f64_score", "cti_f64_norm", "cti_f64_q3", "cti_f64_short", "cti_f64_b2",
                                  "cti_f32_score", "cti_bf16_score"])
def test_compute_token_importance_reference_golden(built_lib, golden, case):
    """Drop-in compute_token_importance vs the reference function's own outputs."""
    from mserve_b200.selection import compute_token_importance
    B, Hq, Hkv, Q, T, D, method, mn = [int(x) for x in golden[f"{case}/meta"]]
    ratio = float(golden[f"{case}/ratio"][0])
    dt = str(golden[f"{case}/dtype"])
    tdt = torch.bfloat16 if "bfloat16" in dt else torch.float32   # f64 inputs are scored in fp32
    q = from_bits(golden[f"{case}/q"], torch.bfloat16 if tdt == torch.bfloat16 else torch.float64).to(tdt)
    k = from_bits(golden[f"{case}/k"], torch.bfloat16 if tdt == torch.bfloat16 else torch.float64).to(tdt)
    mname = ["attention_score", "norm"][method]
    got = compute_token_importance(q.cuda(), k.cuda(), mname, ratio, mn)
    assert got.device.type == "cpu" and got.dtype == torch.int64
    ref = golden[f"{case}/idx"]
    assert tuple(got.shape) == ref.shape
    # oracle fp64 scores of the same inputs decide what counts as a near-tie
    qn, kn = q.double().numpy(), k.double().numpy()
    per = ko.gqa_scores(qn[:, :, -1], kn, method=mname)
    scores = per.sum(axis=1)
    rtol = 2e-2 if tdt == torch.bfloat16 else 1e-5
    got2, ref2 = got.numpy().reshape(B, -1), ref.reshape(B, -1)
    for b in range(B):
        _tie_tolerant_equal(got2[b], ref2[b], scores[b], rtol)


def test_topk_long_context_140k(built_lib):
    """140K candidates: a 4-CTA cluster holding the keys in shared memory."""
    from mserve_b200 import ops
    g = torch.Generator().manual_seed(21)
    rows = torch.randn(3, 140000, generator=g)
    got, cnt = ops.topk(rows.cuda(), top_k=9000, recent=64)
    ref, rcnt = ko.select_topk_window(rows.numpy(), top_k=9000, recent=64)
    got, cnt = got.cpu().numpy(), cnt.cpu().numpy()
    np.testing.assert_array_equal(cnt, rcnt)
    for j in range(3):
        np.testing.assert_array_equal(got[j, :cnt[j]], ref[j])


def test_scores_strided_rows(built_lib):
    """Keys with a token stride of two rows (register-streaming path) and a capacity view."""
    from mserve_b200 import ops
    g = torch.Generator().manual_seed(6)
    B, Hq, Hkv, T, D = 2, 8, 2, 600, 128
    big = torch.randn(B, Hkv, 2 * T, D, generator=g).to(torch.bfloat16).cuda()
    q = torch.randn(B, Hq, D, generator=g).to(torch.bfloat16)
    for k in (big[:, :, ::2, :], big[:, :, :T, :]):
        out = torch.empty(B, Hkv, T, device="cuda")
        ops.score(q.cuda(), ops.strided_rows(k, None), batch=B, kv_heads=Hkv, max_tokens=T, out=out)
        ref = ko.gqa_scores(q.float().numpy(), k.float().cpu().numpy())
        _assert_scores_close(out.cpu().numpy(), ref)


@pytest.mark.parametrize("T", [40000, 70000, 100000, 200000, 400000])   # 1, 2, 4, 8 CTAs; L2 re-read
def test_topk_paths_ties_nan_ragged(built_lib, T):
    """Each top-k path with quantised (tie-heavy) scores, NaN, ragged lengths and per-sequence k."""
    from mserve_b200 import ops
    g = torch.Generator().manual_seed(T)
    B, Hk = 2, 2
    rows = (torch.randn(B * Hk, T, generator=g) * 4).round() * 0.25
    rows[1, 17] = float("nan")
    lens = torch.tensor([T, T // 2 + 3], dtype=torch.int32)
    topk_b = torch.tensor([T // 8, 1000], dtype=torch.int32)
    got, cnt = ops.topk(rows.cuda(), top_k=topk_b.cuda(), recent=128, len_=lens.cuda(), sel_per_batch=Hk)
    ref, rcnt = ko.select_topk_window(rows.numpy(), top_k=topk_b.numpy(), recent=128, lens=lens.numpy(),
                                      sel_per_batch=Hk)
    got, cnt = got.cpu().numpy(), cnt.cpu().numpy()
    np.testing.assert_array_equal(cnt, rcnt)
    for j in range(B * Hk):
        np.testing.assert_array_equal(got[j, :cnt[j]], ref[j])


def test_topk_len_above_len_scalar_is_clamped(built_lib):
    """len[b] beyond len_scalar (which sizes the kernel) is treated as len_scalar."""
    from mserve_b200 import ops
    g = torch.Generator().manual_seed(5)
    rows = torch.randn(2, 5000, generator=g)
    lens = torch.tensor([5000, 3000], dtype=torch.int32)
    got, cnt = ops.topk(rows.cuda(), top_k=100, recent=8, len_=lens.cuda(), len_scalar=2000)
    ref, rcnt = ko.select_topk_window(rows.numpy(), top_k=100, recent=8, lens=[2000, 2000])
    got, cnt = got.cpu().numpy(), cnt.cpu().numpy()
    np.testing.assert_array_equal(cnt, rcnt)
    for j in range(2):
        np.testing.assert_array_equal(got[j, :cnt[j]], ref[j])


def test_topk_summed_rows_cluster_path(built_lib):
    """Few selections that sum several head rows over many tokens (the reference's head mean)
    take the 8-CTA cluster path: exact against the oracle with ties, NaN and ragged lengths."""
    from mserve_b200 import ops
    g = torch.Generator().manual_seed(77)
    B, Hk, T = 3, 4, 20000
    rows = (torch.randn(B * Hk, T, generator=g) * 8).round() * 0.125
    rows[2, 99] = float("nan")
    lens = torch.tensor([T, 15000, 9000], dtype=torch.int32)
    topk_b = torch.tensor([3000, 1, 4321], dtype=torch.int32)
    got, cnt = ops.topk(rows.cuda(), top_k=topk_b.cuda(), recent=64, len_=lens.cuda(), rows_per_sel=Hk,
                        sel_per_batch=1, scale=1.0 / 28)
    ref, rcnt = ko.select_topk_window(rows.numpy(), top_k=topk_b.numpy(), recent=64, lens=lens.numpy(),
                                      rows_per_sel=Hk, sel_per_batch=1, scale=np.float32(1.0 / 28))
    got, cnt = got.cpu().numpy(), cnt.cpu().numpy()
    np.testing.assert_array_equal(cnt, rcnt)
    for j in range(B):
        np.testing.assert_array_equal(got[j, :cnt[j]], ref[j])


def _run_topk_exact(rows: torch.Tensor, K: int, R: int):
    from mserve_b200 import ops
    got, cnt = ops.topk(rows.cuda(), top_k=K, recent=R)
    ref, rcnt = ko.select_topk_window(rows.numpy(), top_k=K, recent=R)
    got, cnt = got.cpu().numpy(), cnt.cpu().numpy()
    np.testing.assert_array_equal(cnt, rcnt)
    for j in range(rows.shape[0]):
        np.testing.assert_array_equal(got[j, :cnt[j]], ref[j])


@pytest.mark.parametrize("T", [16000, 70000, 140000, 300000])   # 1, 2, 4 and 8 CTAs per selection
@pytest.mark.parametrize("stop", ["digit0", "digit1"])
def test_topk_stops_at_a_full_bin(built_lib, T, stop):
    """Selections whose k-th key sits in a bin that is selected in full, so the radix passes stop
    after the first (digit0) or the second (digit1) digit: exact against the oracle."""
    g = torch.Generator().manual_seed(T + (stop == "digit1"))
    S, K, R = 3, T // 10, 32
    rows = torch.rand(S, T, generator=g) * 2 - 1                      # [-1, 1): below every selected key
    for j in range(S):
        top = torch.randperm(T - R, generator=g)[:K]
        if stop == "digit0":
            # all K selected keys in one 12-bit bin: [1024, 1152)
            rows[j, top] = 1024 + 128 * torch.rand(K, generator=g) * 0.999
        else:
            # K - 3 keys far above; three equal keys at 1.6 (24-bit bin full); the rest of the
            # candidates share 1.6's 12-bit bin [1.5, 1.625) below it, or lie in [-1, 1)
            rows[j, top[:K - 3]] = 2048 + 2048 * torch.rand(K - 3, generator=g) * 0.999
            rows[j, top[K - 3:]] = 1.6
            same_bin = torch.randperm(T - R, generator=g)[: T // 4]
            same_bin = same_bin[~torch.isin(same_bin, top)]
            rows[j, same_bin] = 1.5 + 0.09 * torch.rand(len(same_bin), generator=g)
    _run_topk_exact(rows, K, R)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("method", [0, 1])
def test_scores_independent_of_token_stride(built_lib, dtype, D, method):
    """Keys with rows back to back and the same keys at a two-row token stride give
    bit-identical scores: paged with scattered and unmapped pages and ragged lengths, and
    strided (a capacity view)."""
    from mserve_b200 import ops
    g = torch.Generator().manual_seed(D + method)
    dev = torch.device("cuda")
    B, Hq, Hkv, ps, maxp = 3, 12, 4, 16, 40
    P = B * maxp
    q = torch.randn(B, Hq, D, generator=g).to(dtype).to(dev)
    pool = torch.randn(P, Hkv, ps, D, generator=g).to(dtype)
    perm = torch.randperm(P, generator=g).to(torch.int32).view(B, maxp)
    perm[1, 7] = -1                                                   # an unmapped page: -inf scores
    lens = torch.tensor([maxp * ps, 333, 17], dtype=torch.int32).to(dev)
    T = maxp * ps
    wide = torch.zeros(P, Hkv, ps, 2, D, dtype=dtype)
    wide[:, :, :, 0] = pool
    outs = []
    for k_pool in (pool.to(dev), wide.to(dev).view(P, Hkv, 2 * ps, D)[:, :, ::2]):
        out = torch.full((B, Hkv, T), float("nan"), device=dev)
        rows = ops.paged_rows(k_pool, None, perm.to(dev), len_=lens)
        ops.score(q, rows, batch=B, kv_heads=Hkv, max_tokens=T, out=out, method=method)
        outs.append(out.cpu())
    assert torch.equal(outs[0].isnan(), outs[1].isnan())
    assert torch.equal(torch.nan_to_num(outs[0], nan=7.0), torch.nan_to_num(outs[1], nan=7.0))
    assert torch.isinf(outs[0][1, :, 7 * ps:8 * ps]).all()
    # strided [B, Hkv, T, D] (capacity view) against the same keys at a two-row stride
    k = torch.randn(B, Hkv, 2 * T, D, generator=g).to(dtype).to(dev)
    k2 = torch.zeros(B, Hkv, T, 2, D, dtype=dtype, device=dev)
    k2[:, :, :, 0] = k[:, :, :T]
    res = []
    for kv in (k[:, :, :T], k2.view(B, Hkv, 2 * T, D)[:, :, ::2]):
        out = torch.empty(B, Hkv, T, device=dev)
        ops.score(q, ops.strided_rows(kv, None), batch=B, kv_heads=Hkv, max_tokens=T, out=out, method=method)
        res.append(out.cpu())
    assert torch.equal(res[0], res[1])
    ops.check_status(dev, "scores at two token strides")
