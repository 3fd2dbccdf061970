"""The prefill image-token filter on the GPU (mskv_image_filter via selection.dual_attention_filter).

Against the reference's own outputs on the golden blocks (kept sets equal except next to a
threshold), and against the oracle, which sums in the kernels' fixed order and rounds the same
stages: the kept sets are identical.
"""
import numpy as np
import pytest
import torch

from oracle import kv_oracle as ko
from test_filter_golden import (CASES, FIX, ITHR_CASES, ITHR_COLUMNS, STAGE_RTOL, assert_sets_match, load_case,
                                run_oracle)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def fix():
    return np.load(FIX)


@pytest.mark.parametrize("name", CASES)
def test_filter_matches_reference_and_oracle(built_lib, fix, name):
    from mserve_b200.selection import dual_attention_filter
    attn, c = load_case(fix, name)
    got, text_seq = dual_attention_filter(attn.cuda(), c["start"], c["img"], c["gthr"], c["ithr"], use_fp16=c["fp16"])
    assert got.is_cuda and got.dtype == torch.int64
    assert text_seq == int(fix[f"{name}/text_seq"][0])
    got = got.cpu().numpy()
    kept, _, attn_sum, text_max, thr = run_oracle(attn, c)
    np.testing.assert_array_equal(got, kept)
    assert_sets_match(got, fix[f"{name}/idx"], attn_sum, text_max, thr, c["ithr"], 4 * STAGE_RTOL[c["stage"]])


@pytest.mark.parametrize("name", ITHR_CASES)
def test_filter_rounds_individual_threshold(built_lib, fix, name):
    """The kernel rounds individual_thr to the stage dtype as torch does: the reference's kept set
    exactly, the column sitting on the rounded threshold included."""
    from mserve_b200.selection import dual_attention_filter
    attn, c = load_case(fix, name)
    got, _ = dual_attention_filter(attn.cuda(), c["start"], c["img"], c["gthr"], c["ithr"], use_fp16=c["fp16"])
    got = got.cpu().numpy()
    assert [col in set(got.tolist()) for col in ITHR_COLUMNS] == [True, False, True]
    np.testing.assert_array_equal(got, fix[f"{name}/idx"])


def _probabilities(H, T, seed):
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(1, H, T, T, generator=g) * 1.5 + torch.randn(T, generator=g) * 2.5
    return torch.softmax(logits, dim=-1)


@pytest.mark.parametrize("dtype,use_fp16,text", [(torch.float32, False, 100), (torch.float32, True, 100),
                                                 (torch.bfloat16, False, 33), (torch.float16, False, 7),
                                                 (torch.float32, False, 1000)])
def test_filter_image_sized(built_lib, dtype, use_fp16, text):
    """A 36 x 36 token image (1296 tokens) behind 15 system tokens, 28 heads."""
    from mserve_b200.selection import dual_attention_filter
    H, start, img = 28, 15, 1296
    attn = _probabilities(H, start + img + text, seed=text).to(dtype)
    got, ts = dual_attention_filter(attn.cuda(), start, img, 0.0005, 0.01, use_fp16=use_fp16)
    assert ts == text
    stage = "f16" if (use_fp16 or dtype == torch.float16) else ("bf16" if dtype == torch.bfloat16 else "f32")
    kept, *_ = ko.dual_attention_filter(attn.float().numpy(), start, img, 0.0005, 0.01, stage=stage)
    np.testing.assert_array_equal(got.cpu().numpy(), kept)
    assert 0 < kept.size < img


def test_filter_strided_view_and_edges(built_lib):
    from mserve_b200 import ops
    from mserve_b200.selection import dual_attention_filter
    H, start, img, text = 5, 4, 1000, 9
    T = start + img + text
    attn = _probabilities(H, T, seed=3)
    # a [B, H, T, T] view whose key axis is not contiguous
    attn_t = attn.transpose(2, 3).contiguous().transpose(2, 3).cuda()
    got, _ = dual_attention_filter(attn_t, start, img, 0.002, 0.01)
    kept, *_ = ko.dual_attention_filter(attn.numpy(), start, img, 0.002, 0.01)
    np.testing.assert_array_equal(got.cpu().numpy(), kept)
    assert 0 < got.numel() < img
    # no image tokens: nothing kept
    empty, ts = dual_attention_filter(attn.cuda(), start, 0, 0.002, 0.01)
    assert empty.numel() == 0 and ts == T - start
    # on a side stream, without synchronising first
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    idx, count = ops.image_filter(attn[0].cuda(), img_start=start, img_seq=img, text_start=start + img, text_seq=text,
                                  global_thr=0.002, individual_thr=0.01, stream=s)
    s.synchronize()
    np.testing.assert_array_equal(idx[:int(count.item())].cpu().numpy(), kept)
    with pytest.raises(ValueError):
        ops.image_filter(attn[0].cuda(), img_start=0, img_seq=T, text_start=T, text_seq=0, global_thr=1.0,
                         individual_thr=0.0)
    with pytest.raises(ValueError):
        ops.image_filter(attn[0].cuda(), img_start=T - 3, img_seq=10, text_start=0, text_seq=2, global_thr=1.0,
                         individual_thr=0.0)
    with pytest.raises(ValueError):
        ops.image_filter(attn[0].cuda().half(), img_start=0, img_seq=4, text_start=4, text_seq=2, global_thr=1.0,
                         individual_thr=0.0, round_f16=True)


@pytest.mark.parametrize("H,text,img,dtype", [
    (40, 33, 2500, torch.float32),     # 40 heads: two full head batches and a remainder; 3 rounds
    (3, 1, 3000, torch.bfloat16),      # one text row: 32-thread CTAs, 94 compaction rounds
    (2, 2, 70000, torch.float32),      # more tiles than the last CTA keeps in shared memory
])
def test_filter_block_edges(built_lib, H, text, img, dtype):
    """mskv_image_filter on a [H, text, img] block at the edges of its launch shapes, against
    the oracle's block form (same stage rounding and summation order): identical kept sets."""
    from mserve_b200 import ops
    g = torch.Generator().manual_seed(H * 1000 + text)
    # a third of the columns at twice the scale (kept by their sum); a tenth at a small scale
    # with one large element (kept, where the text has several rows, by their maximum alone)
    order = torch.randperm(img, generator=g)
    scale = torch.ones(img)
    scale[order[:img // 3]] = 2.0
    spikes = order[img // 3:img // 3 + img // 10]
    scale[spikes] = 0.3
    block = torch.rand(H, text, img, generator=g) * scale
    block[torch.randint(H, (spikes.numel(),), generator=g), torch.randint(text, (spikes.numel(),), generator=g),
          spikes] += (1 + torch.rand(spikes.numel(), generator=g)) * 2 * H
    block = block.to(dtype)
    stage = "bf16" if dtype == torch.bfloat16 else "f32"
    _, _, text_max, _ = ko.image_filter_block(block.float().numpy(), 0.0, 0.0, stage)
    gthr, ithr = 1.0 / img, float(np.quantile(text_max, 0.9))   # the mean share; the top tenth's maxima
    kept, attn_sum, _, thr = ko.image_filter_block(block.float().numpy(), gthr, ithr, stage)
    assert 0 < kept.size < img
    idx, count = ops.image_filter(block.cuda(), img_start=0, img_seq=img, text_start=0, text_seq=text,
                                  global_thr=gthr, individual_thr=ithr)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(idx[:int(count.item())].cpu().numpy(), kept)
