"""The prefill image-token filter on the GPU (mskv_image_filter via selection.dual_attention_filter).

Against the reference's own outputs on the golden blocks (kept sets equal except next to a
threshold), and against the oracle, which accumulates in the kernel's order (heads, then text
rows), exactly wherever no token sits within a hair of a threshold.
"""
import numpy as np
import pytest
import torch

from oracle import kv_oracle as ko
from test_filter_golden import CASES, FIX, assert_sets_match, load_case

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
    a = attn.half().float() if c["fp16"] else attn.float()
    kept, _, attn_sum, text_max, total = ko.dual_attention_filter(a.numpy(), c["start"], c["img"], c["gthr"], c["ithr"])
    rtol = 1e-5 if not (c["bf16"] or c["fp16"]) else 1e-2
    assert_sets_match(got, fix[f"{name}/idx"], attn_sum, text_max, total, c["gthr"], c["ithr"], rtol)
    assert_sets_match(got, kept, attn_sum, text_max, total, c["gthr"], c["ithr"], 1e-6)


def test_filter_strided_view_and_edges(built_lib):
    from mserve_b200 import ops
    from mserve_b200.selection import dual_attention_filter
    g = torch.Generator().manual_seed(3)
    H, start, img, text = 5, 4, 1000, 9
    T = start + img + text
    logits = torch.randn(1, H, T, T, generator=g) * 1.5 + torch.randn(T, generator=g) * 2.5
    attn = torch.softmax(logits, dim=-1)
    # a [B, H, T, T] view whose key axis is not contiguous
    attn_t = attn.transpose(2, 3).contiguous().transpose(2, 3).cuda()
    got, _ = dual_attention_filter(attn_t, start, img, 0.002, 0.01)
    kept, _, s, m, total = ko.dual_attention_filter(attn.numpy(), start, img, 0.002, 0.01)
    assert_sets_match(got.cpu().numpy(), kept, s, m, total, 0.002, 0.01, 1e-6)
    assert 0 < got.numel() < img
    # no image tokens: nothing kept
    empty, ts = dual_attention_filter(attn.cuda(), start, 0, 0.002, 0.01)
    assert empty.numel() == 0 and ts == T - start
    with pytest.raises(ValueError):
        ops.image_filter(attn[0].cuda(), img_start=0, img_seq=T, text_start=T, text_seq=0, global_thr=1.0,
                         individual_thr=0.0)
    with pytest.raises(ValueError):
        ops.image_filter(attn[0].cuda(), img_start=T - 3, img_seq=10, text_start=0, text_seq=2, global_thr=1.0,
                         individual_thr=0.0)
