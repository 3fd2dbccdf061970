"""The prefill image-token filter oracle against the reference's own outputs (CPU).

tests/golden/filter_vectors.npz holds the text x image block of batch 0, the arguments, and what
MServe's dual_attention_filter returned for it (tests/golden/make_filter_golden.py).  For fp32
blocks the oracle's per-token column sums and maxima equal torch's to within 1e-6 (summation
order) and the kept sets are equal except for tokens within a hair of a threshold; for bf16 blocks and the fp16 rounding mode, where the reference averages in low
precision, the sets are equal except within 1% of a threshold.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import kv_oracle as ko

FIX = Path(__file__).resolve().parent / "golden" / "filter_vectors.npz"
CASES = ["thr_small", "heads28", "defaults", "bf16", "fp16_round"]


def load_case(fix, name):
    H, start, img, text, T, fp16, bf16 = (int(x) for x in fix[f"{name}/meta"])
    gthr, ithr = (float(x) for x in fix[f"{name}/thr"])
    blk = fix[f"{name}/block"]
    block = torch.from_numpy(blk.view(np.int16)).view(torch.bfloat16) if bf16 else torch.from_numpy(blk)
    attn = torch.zeros(1, H, T, T, dtype=block.dtype)
    attn[0, :, start + img:start + img + text, start:start + img] = block
    return attn, dict(H=H, start=start, img=img, text=text, gthr=gthr, ithr=ithr, fp16=bool(fp16), bf16=bool(bf16))


def near_threshold(attn_sum, text_max, total, gthr, ithr, rtol):
    """Tokens whose drop decision could flip under a relative perturbation of rtol."""
    g = total * gthr
    return (np.abs(attn_sum - g) <= rtol * abs(g) + 1e-30) | (np.abs(text_max - ithr) <= rtol * abs(ithr) + 1e-30)


def assert_sets_match(got, ref, attn_sum, text_max, total, gthr, ithr, rtol):
    diff = set(got.tolist()) ^ set(ref.tolist())
    if diff:
        near = near_threshold(attn_sum, text_max, total, gthr, ithr, rtol)
        bad = [j for j in diff if not near[j]]
        assert not bad, f"{len(bad)} tokens differ away from the thresholds"
    assert list(got) == sorted(got)


@pytest.fixture(scope="module")
def fix():
    return np.load(FIX)


@pytest.mark.parametrize("name", CASES)
def test_filter_oracle_matches_reference(fix, name):
    attn, c = load_case(fix, name)
    a = attn.half().float() if c["fp16"] else attn.float()
    kept, text_seq, attn_sum, text_max, total = ko.dual_attention_filter(
        a.numpy(), c["start"], c["img"], c["gthr"], c["ithr"])
    assert text_seq == int(fix[f"{name}/text_seq"][0])
    ref = fix[f"{name}/idx"]
    if not c["bf16"] and not c["fp16"]:
        # fp32: the column sums and maxima differ from torch's by summation order only (torch's
        # CPU reductions group the heads and the text rows their own way)
        np.testing.assert_allclose(text_max, fix[f"{name}/text_max"], rtol=1e-6, atol=0)
        np.testing.assert_allclose(attn_sum, fix[f"{name}/attn_sum"], rtol=1e-6, atol=0)
        assert_sets_match(kept, ref, attn_sum, text_max, total, c["gthr"], c["ithr"], 1e-5)
    else:
        assert_sets_match(kept, ref, attn_sum, text_max, total, c["gthr"], c["ithr"], 1e-2)
