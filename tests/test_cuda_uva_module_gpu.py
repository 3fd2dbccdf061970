"""The `cuda_uva` module by its own name: an unmodified `import cuda_uva` (the import of
qwen-eljrte/Qwen_Transformer/kv_cache.py:512 and qwen-eljrte/benchmark_kv_transfer.py:36-43)
resolves to the torch extension built from mserve_b200/torch_ext/cuda_uva.cpp once that
directory is on sys.path, and its uva_gather is bit-exact with the oracle's index_select
restatement (oracle/kv_oracle.py:index_select_gather) for every element type and index form.
"""
import sys

import numpy as np
import pytest
import torch

from conftest import to_numpy_bits
from oracle import kv_oracle as ko

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda_uva(built_lib):
    from mserve_b200 import build
    ext = build.build_torch_ext()
    if str(ext.parent) not in sys.path:
        sys.path.insert(0, str(ext.parent))
    import cuda_uva as mod       # the reference's import, unmodified
    assert mod.__file__ == str(ext)
    return mod


def _pinned(shape, dtype, g):
    x = torch.randn(*shape, generator=g)
    return (x * 4).to(dtype).pin_memory() if dtype.is_floating_point and dtype.itemsize == 1 else x.to(dtype).pin_memory()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32, torch.float64, torch.float8_e4m3fn,
                                   torch.float8_e5m2])
@pytest.mark.parametrize("B,H,T,D,S,order", [(1, 8, 8192, 128, 2048, "random"),   # the harness default shape
                                             (2, 4, 1000, 64, 333, "sorted"),
                                             (1, 3, 77, 80, 200, "duplicates")])
def test_module_gather_bit_exact(cuda_uva, dtype, B, H, T, D, S, order):
    g = torch.Generator().manual_seed(T + S)
    k, v = _pinned((B, H, T, D), dtype, g), _pinned((B, H, T, D), dtype, g)
    if order == "duplicates":
        idx = torch.randint(0, T, (S,), generator=g)
    else:
        idx = torch.randperm(T, generator=g)[:S]
        if order == "sorted":
            idx = idx.sort().values
    k_out, v_out = cuda_uva.uva_gather(k, v, idx, B, H, T, D)
    torch.cuda.synchronize()
    assert k_out.is_cuda and k_out.shape == (B, H, S, D) and k_out.dtype == dtype
    ek, ev = ko.index_select_gather(to_numpy_bits(k), to_numpy_bits(v), idx.numpy())
    np.testing.assert_array_equal(to_numpy_bits(k_out), ek)
    np.testing.assert_array_equal(to_numpy_bits(v_out), ev)
    # the same through device-resident indices
    k2, v2 = cuda_uva.uva_gather(k, v, idx.cuda(), B, H, T, D)
    torch.cuda.synchronize()
    cuda_uva.check_errors()
    assert torch.equal(to_numpy_bits_t(k2), to_numpy_bits_t(k_out)) and torch.equal(to_numpy_bits_t(v2), to_numpy_bits_t(v_out))


def to_numpy_bits_t(t):
    return torch.from_numpy(to_numpy_bits(t))


def test_module_errors(cuda_uva):
    g = torch.Generator().manual_seed(1)
    k = torch.randn(1, 2, 64, 32, generator=g).to(torch.bfloat16)
    with pytest.raises(RuntimeError, match="k_in must be pinned memory for UVA"):
        cuda_uva.uva_gather(k, k.pin_memory(), torch.tensor([1, 2]), 1, 2, 64, 32)
    kp = k.pin_memory()
    with pytest.raises(RuntimeError, match="out of range"):
        cuda_uva.uva_gather(kp, kp, torch.tensor([0, 64]), 1, 2, 64, 32)
    with pytest.raises(RuntimeError, match="not implemented for"):
        cuda_uva.uva_gather(kp.to(torch.int16).pin_memory(), kp.to(torch.int16).pin_memory(), torch.tensor([0]),
                            1, 2, 64, 32)
    # a device index list is checked on the device: the row is zero-filled and reported
    ko_, _ = cuda_uva.uva_gather(kp, kp, torch.tensor([3, 64], device="cuda"), 1, 2, 64, 32)
    with pytest.raises(RuntimeError, match="out of range"):
        cuda_uva.check_errors()
    assert torch.count_nonzero(ko_[:, :, 1].float()) == 0
    assert torch.equal(ko_[:, :, 0].cpu(), k[:, :, 3])
    cuda_uva.check_errors()          # the status word was cleared
