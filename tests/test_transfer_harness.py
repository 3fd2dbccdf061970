"""The transfer harness's index generators (CPU only).  generate_scattered_indices must give
the reference's indices for the same seed (golden vectors from the reference's own function)."""
import numpy as np
import pytest
import torch

from mserve_b200.benchmark_kv_transfer import generate_scattered_indices, structured_indices


@pytest.mark.parametrize("key,args", [("scatter/8192_2048_42", (8192, 2048, 42)), ("scatter/4096_100_7", (4096, 100, 7))])
def test_scattered_indices_match_reference(golden, key, args):
    np.testing.assert_array_equal(generate_scattered_indices(*args).numpy(), golden[key])


@pytest.mark.parametrize("run", [1, 16, 64])
def test_structured_indices(run):
    g = torch.Generator().manual_seed(4)
    idx = structured_indices(131072, 6553, run, g)
    assert len(idx) == len(torch.unique(idx)) and (idx[1:] > idx[:-1]).all()
    assert idx.min() >= 0 and idx.max() < 131072
    if run > 1:   # whole runs of `run` consecutive tokens
        starts = idx[(idx % run) == 0]
        assert len(starts) >= len(idx) // run - 1
