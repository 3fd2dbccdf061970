"""The prefill image-token filter oracle against the reference's own outputs (CPU).

tests/golden/filter_vectors.npz holds the text x image block of batch 0, the arguments, and what
MServe's dual_attention_filter returned for it (tests/golden/make_filter_golden.py).  For fp32
blocks the oracle's per-token column sums and maxima equal torch's to within 1e-6 (summation
order); for bf16 blocks and the fp16 rounding mode, where every stage is rounded to the 16-bit
dtype, to within one unit in the last place of that dtype.  The kept sets are equal except for
tokens next to a threshold (none in these fixtures).
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import kv_oracle as ko

FIX = Path(__file__).resolve().parent / "golden" / "filter_vectors.npz"
CASES = ["thr_small", "heads28", "defaults", "bf16", "fp16_round", "callsite", "ithr_bf16", "ithr_f16",
         "ithr_fp16_mode"]
# cases whose columns 10, 50 and 120 hold, in one text row, the individual threshold rounded to
# the stage dtype, the value below it and the value above it (tests/golden/make_filter_golden.py)
ITHR_CASES = ["ithr_bf16", "ithr_f16", "ithr_fp16_mode"]
ITHR_COLUMNS = (10, 50, 120)
# one unit in the last place, relative: fp32 order effects / fp16 / bf16
STAGE_RTOL = {"f32": 1e-6, "f16": 2.0 ** -10, "bf16": 2.0 ** -7}


def load_case(fix, name):
    H, start, img, text, T, fp16, bf16, f16 = (int(x) for x in fix[f"{name}/meta"])
    gthr, ithr = (float(x) for x in fix[f"{name}/thr"])
    blk = fix[f"{name}/block"]
    block = torch.from_numpy(blk.view(np.int16)).view(torch.bfloat16) if bf16 else torch.from_numpy(blk)
    attn = torch.zeros(1, H, T, T, dtype=block.dtype)
    attn[0, :, start + img:start + img + text, start:start + img] = block
    stage = "f16" if (fp16 or f16) else ("bf16" if bf16 else "f32")
    return attn, dict(H=H, start=start, img=img, text=text, gthr=gthr, ithr=ithr, fp16=bool(fp16), bf16=bool(bf16),
                      stage=stage)


def near_threshold(attn_sum, text_max, thr, ithr, rtol):
    """Tokens whose drop decision could flip under a relative perturbation of rtol."""
    return (np.abs(attn_sum - thr) <= rtol * abs(thr) + 1e-30) | (np.abs(text_max - ithr) <= rtol * abs(ithr) + 1e-30)


def assert_sets_match(got, ref, attn_sum, text_max, thr, ithr, rtol):
    diff = set(got.tolist()) ^ set(ref.tolist())
    if diff:
        near = near_threshold(attn_sum, text_max, thr, ithr, rtol)
        bad = [j for j in diff if not near[j]]
        assert not bad, f"{len(bad)} tokens differ away from the thresholds"
    assert list(got) == sorted(got)


def run_oracle(attn, c):
    return ko.dual_attention_filter(attn.float().numpy(), c["start"], c["img"], c["gthr"], c["ithr"], stage=c["stage"])


@pytest.fixture(scope="module")
def fix():
    return np.load(FIX)


@pytest.mark.parametrize("name", CASES)
def test_filter_oracle_matches_reference(fix, name):
    attn, c = load_case(fix, name)
    kept, text_seq, attn_sum, text_max, thr = run_oracle(attn, c)
    assert text_seq == int(fix[f"{name}/text_seq"][0])
    rtol = STAGE_RTOL[c["stage"]]
    np.testing.assert_allclose(text_max, fix[f"{name}/text_max"], rtol=rtol, atol=0)
    np.testing.assert_allclose(attn_sum, fix[f"{name}/attn_sum"], rtol=rtol, atol=0)
    assert_sets_match(kept, fix[f"{name}/idx"], attn_sum, text_max, thr, c["ithr"], 4 * rtol)


@pytest.mark.parametrize("name", ITHR_CASES)
def test_filter_oracle_rounds_individual_threshold(fix, name):
    """A column whose maximum equals the threshold rounded to the stage dtype is kept, exactly as
    the reference keeps it; the one just below is dropped (no tolerance: these columns sit on
    the threshold by construction)."""
    attn, c = load_case(fix, name)
    kept, *_ = run_oracle(attn, c)
    ref = set(fix[f"{name}/idx"].tolist())
    assert [col in ref for col in ITHR_COLUMNS] == [True, False, True]
    assert [col in set(kept.tolist()) for col in ITHR_COLUMNS] == [True, False, True]
    np.testing.assert_array_equal(kept, fix[f"{name}/idx"])


def test_stage_rounding():
    x = np.array([1.0, 1.00390625, 1.01171875, 1.0 + 2.0 ** -12, 3.0e-5, 0.1], dtype=np.float32)
    # bf16 keeps 8 significant bits, nearest even: 1 + 2^-8 is a tie that rounds down to 1
    np.testing.assert_array_equal(ko._stage(x, "bf16"), torch.from_numpy(x).bfloat16().float().numpy())
    np.testing.assert_array_equal(ko._stage(x, "f16"), torch.from_numpy(x).half().float().numpy())
    np.testing.assert_array_equal(ko._stage(x, "f32"), x)


def test_empty_image_and_defaults():
    g = np.random.default_rng(0)
    attn = g.random((1, 2, 20, 20), dtype=np.float32)
    kept, text_seq, *_ = ko.dual_attention_filter(attn, 3, 0)
    assert kept.size == 0 and text_seq == 17
    # global_thr 1 and individual_thr 0 (the defaults) drop nothing: max < 0 never holds
    kept, *_ = ko.dual_attention_filter(attn, 3, 10)
    assert kept.tolist() == list(range(10))
