"""The reference's own UVA gather kernel against mskv_uva_gather, bit for bit.

oracle/build_ref.py compiles qwen-eljrte/cuda_uva_kernel.cpp unmodified (as CUDA, for sm_100a)
into oracle/_ref/cuda_uva_ref.so.  Both gathers run on the same pinned [B, H, T, D] cache and
the same index list; the outputs must be identical bit for bit.

The reference kernel dereferences every pointer it is given on the device, the index list
included (qwen-eljrte/cuda_uva_kernel.cpp:36, a CPU tensor).  That is valid only for page-locked
host memory, which unified addressing maps at the same address on the device.  The test pins
K, V and the indices and, before any launch, checks that each of them is device-accessible at
exactly its host address; otherwise it skips rather than run the reference kernel.
"""
import ctypes as C

import pytest
import torch

from oracle import build_ref

pytestmark = pytest.mark.gpu


def _same_address_on_device(t: torch.Tensor) -> bool:
    from mserve_b200 import _lib
    p = C.c_void_p()
    rc = _lib.lib().mskv_device_view(C.c_void_p(t.data_ptr()), C.byref(p))
    return rc == _lib.MSKV_OK and p.value == t.data_ptr()


@pytest.fixture(scope="module")
def ref_module():
    mod = build_ref.load()
    if mod is None:
        pytest.skip("the reference extension is not built (oracle/build_ref.py)")
    return mod


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32, torch.float64])
@pytest.mark.parametrize("B,H,T,D,S,order", [(1, 4, 32768, 128, 4096, "sorted"),   # one layer of the 7B cache
                                             (1, 8, 8192, 128, 2048, "shuffled"),   # the harness default shape
                                             (2, 3, 1000, 64, 77, "shuffled")])
def test_reference_kernel_bit_exact(built_lib, ref_module, dtype, B, H, T, D, S, order):
    from mserve_b200 import cuda_uva
    g = torch.Generator().manual_seed(T + S)
    k = torch.randn(B, H, T, D, generator=g).to(dtype).pin_memory()
    v = torch.randn(B, H, T, D, generator=g).to(dtype).pin_memory()
    idx = torch.randperm(T, generator=g)[:S]
    if order == "sorted":
        idx = idx.sort().values
    idx = idx.to(torch.int64).pin_memory()
    for t in (k, v, idx):
        if not _same_address_on_device(t):
            pytest.skip("pinned memory is not device-accessible at its host address here")
    rk, rv = ref_module.uva_gather(k, v, idx, B, H, T, D)
    torch.cuda.synchronize()
    ok, ov = cuda_uva.uva_gather(k, v, idx, B, H, T, D)
    torch.cuda.synchronize()
    bits = {1: torch.uint8, 2: torch.int16, 4: torch.int32, 8: torch.int64}[k.element_size()]
    assert torch.equal(rk.view(bits), ok.view(bits))
    assert torch.equal(rv.view(bits), ov.view(bits))
    # and both equal the host-side index_select the gather stands for
    assert torch.equal(ok.cpu().view(bits), torch.index_select(k, 2, idx).view(bits))
