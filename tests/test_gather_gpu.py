"""Parity of the sm_100a gather (mskv_uva_gather / mskv_gather) with the oracle: bit-exact.

Reference semantics: out[b,h,s,:] = in[b,h,indices[s],:] (qwen-eljrte/cuda_uva_kernel.cpp:29-44,
qwen-eljrte/Qwen_Transformer/kv_cache.py:597-599).
"""
import zlib

import numpy as np
import pytest
import torch

from conftest import from_bits, to_numpy_bits
from oracle import kv_oracle as ko

pytestmark = pytest.mark.gpu


def _pinned_randn(shape, dtype, gen):
    x = torch.randn(*shape, generator=gen, dtype=torch.float32)
    if dtype in (torch.float8_e4m3fn, torch.float8_e5m2):
        x = x.clamp(-200, 200)
    return x.to(dtype).pin_memory()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32, torch.float64,
                                   torch.float8_e4m3fn, torch.float8_e5m2])
@pytest.mark.parametrize("shape", [(1, 8, 8192, 128, 2048), (2, 3, 100, 7, 33), (1, 1, 5, 1, 5),
                                   (3, 2, 300, 64, 1), (1, 4, 1000, 128, 999)])
def test_uva_gather_bit_exact(built_lib, dtype, shape):
    from mserve_b200 import cuda_uva
    B, H, T, D, S = shape
    g = torch.Generator().manual_seed(zlib.crc32(repr((str(dtype), shape)).encode()))
    k = _pinned_randn((B, H, T, D), dtype, g)
    v = _pinned_randn((B, H, T, D), dtype, g)
    idx = torch.randint(0, T, (S,), generator=g, dtype=torch.int64)   # duplicates, any order
    ko_, vo_ = cuda_uva.uva_gather(k, v, idx, B, H, T, D)
    torch.cuda.synchronize()
    ek, ev = ko.index_select_gather(to_numpy_bits(k), to_numpy_bits(v), idx.numpy())
    assert ko_.shape == (B, H, S, D) and ko_.dtype == dtype and ko_.is_cuda
    np.testing.assert_array_equal(to_numpy_bits(ko_), ek)
    np.testing.assert_array_equal(to_numpy_bits(vo_), ev)
    cuda_uva.check_errors()


def test_uva_gather_reference_golden(built_lib, golden):
    """Same inputs as the reference's CPUKVCache.get_sparse_async run (tests/golden)."""
    from mserve_b200 import cuda_uva
    k = from_bits(golden["sparse/k"], torch.bfloat16).pin_memory()
    v = from_bits(golden["sparse/v"], torch.bfloat16).pin_memory()
    idx = torch.from_numpy(golden["sparse/idx"])
    B, H, T, D = k.shape
    ko_, vo_ = cuda_uva.uva_gather(k, v, idx, B, H, T, D)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(to_numpy_bits(ko_), golden["sparse/k_sel"].view(np.int16))
    np.testing.assert_array_equal(to_numpy_bits(vo_), golden["sparse/v_sel"].view(np.int16))


def test_uva_gather_errors(built_lib):
    from mserve_b200 import cuda_uva
    k = torch.randn(1, 2, 10, 8).to(torch.bfloat16)
    with pytest.raises(RuntimeError, match="pinned"):
        cuda_uva.uva_gather(k, k, torch.tensor([0, 1]), 1, 2, 10, 8)
    kp = k.pin_memory()
    with pytest.raises(RuntimeError, match="out of range"):
        cuda_uva.uva_gather(kp, kp, torch.tensor([0, 10]), 1, 2, 10, 8)
    with pytest.raises(RuntimeError, match="not implemented"):
        ki = torch.zeros(1, 2, 10, 8, dtype=torch.int32).pin_memory()
        cuda_uva.uva_gather(ki, ki, torch.tensor([0]), 1, 2, 10, 8)
    # device indices are checked on the device: the bad row is zero-filled and reported
    idx = torch.tensor([3, 10, 2], device="cuda")
    ko_, _ = cuda_uva.uva_gather(kp, kp, idx, 1, 2, 10, 8)
    with pytest.raises(RuntimeError, match="out of range"):
        cuda_uva.check_errors()
    out = ko_.cpu()
    assert torch.equal(out[:, :, 0], kp[:, :, 3]) and torch.equal(out[:, :, 2], kp[:, :, 2])
    assert (out[:, :, 1].float() == 0).all()
    cuda_uva.check_errors()   # cleared


def test_uva_gather_empty(built_lib):
    from mserve_b200 import cuda_uva
    k = torch.randn(1, 2, 10, 8).to(torch.bfloat16).pin_memory()
    ko_, vo_ = cuda_uva.uva_gather(k, k, torch.zeros(0, dtype=torch.int64), 1, 2, 10, 8)
    assert ko_.shape == (1, 2, 0, 8) and vo_.shape == (1, 2, 0, 8)


@pytest.mark.parametrize("index_dtype", [torch.int32, torch.int64])
@pytest.mark.parametrize("layout", ["per_head", "per_seq", "shared"])
def test_gather_segments_ring_counts(built_lib, index_dtype, layout):
    """Per-segment index lists, ragged counts, a wrapped ring store with per-sequence length."""
    from mserve_b200 import ops
    g = torch.Generator().manual_seed(5)
    B, H, C, D, S = 3, 4, 96, 128, 40
    k = ops.host_empty((B, H, C, D), torch.bfloat16)
    v = ops.host_empty((B, H, C, D), torch.bfloat16)
    k.copy_(torch.randn(B, H, C, D, generator=g).to(torch.bfloat16))
    v.copy_(torch.randn(B, H, C, D, generator=g).to(torch.bfloat16))
    lens = torch.tensor([96, 50, 70], dtype=torch.int32)
    start = torch.tensor([10, 90, 0], dtype=torch.int32)
    shape = {"per_head": (B, H, S), "per_seq": (B, S), "shared": (S,)}[layout]
    idx = torch.randint(0, 50, shape, generator=g).to(index_dtype)
    counts = torch.randint(0, S + 1, (B, H), generator=g, dtype=torch.int32)
    dev = torch.device("cuda")
    ko_ = torch.zeros(B, H, S, D, dtype=torch.bfloat16, device=dev)
    vo_ = torch.zeros_like(ko_)
    src = ops.strided_rows(k, v, len_=lens.to(dev), ring_start=start.to(dev), ring_cap=C, device=dev)
    ops.gather(src, idx.to(dev).contiguous(), ko_, vo_, batch=B, counts=counts.to(dev))
    ops.check_status(dev)
    ek, ev, mask, oob = ko.gather_segments(to_numpy_bits(k), to_numpy_bits(v), idx.numpy(), counts=counts.numpy(),
                                           lens=lens.numpy(), ring_start=start.numpy(), ring_cap=C)
    assert not oob
    got_k, got_v = to_numpy_bits(ko_), to_numpy_bits(vo_)
    np.testing.assert_array_equal(got_k[mask], ek[mask])
    np.testing.assert_array_equal(got_v[mask], ev[mask])
    assert (got_k[~mask] == 0).all()          # rows past the count are not written


def test_gather_full_7b_layer_4096_of_32768(built_lib):
    """One layer of the CPU-reference gather workload: K,V [32768 tokens, 4 KV heads, 128] bf16,
    4096 sorted unique indices -- bit-exact against index_select."""
    from mserve_b200 import cuda_uva
    g = torch.Generator().manual_seed(0)
    k = torch.randn(1, 4, 32768, 128, generator=g).to(torch.bfloat16).pin_memory()
    v = torch.randn(1, 4, 32768, 128, generator=g).to(torch.bfloat16).pin_memory()
    idx = torch.randperm(32768, generator=torch.Generator().manual_seed(1))[:4096].sort().values
    ko_, vo_ = cuda_uva.uva_gather(k, v, idx, 1, 4, 32768, 128)
    torch.cuda.synchronize()
    ek, ev = ko.index_select_gather(to_numpy_bits(k), to_numpy_bits(v), idx.numpy())
    np.testing.assert_array_equal(to_numpy_bits(ko_), ek)
    np.testing.assert_array_equal(to_numpy_bits(vo_), ev)
