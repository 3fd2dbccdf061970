"""mskv_sparse_attention_noalloc: decode attention for callers that cannot allocate.

Some callers cannot hand the library a workspace: they run where cudaMalloc is forbidden or
unsafe (under an allocator lock, inside another library's memory pool, on a host framework's
allocation-free decode path).  The entry point uses a scratch array built into the library
instead.  This test calls it through the C ABI (ctypes, no Python wrapper) and checks its
output against the regular entry point, mskv_sparse_attention with a workspace, on calls in a
row with different shapes, then checks that a shape one split too large for the array is
refused.  Selections of up to 8 x 4096 rows run the streaming cluster kernel, which needs no
scratch at all; wider ones run the split-sequence kernels, whose partials use the array -- the
widest case here needs all but 2 KB of it, so its far end is written and read.  Both entry
points run the same kernels with the same split of the selected rows, so the outputs must be
bit-identical.  The file is named to be collected last.
"""
import ctypes as C
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _desc(q, k, v, counts, out):
    from mserve_b200._lib import AttnDesc
    from mserve_b200 import ops
    B, Hq, Q, D = q.shape
    Hk, S = k.shape[1], k.shape[2]
    es = q.element_size()
    d = AttnDesc()
    d.q = q.data_ptr()
    d.q_stride_b, d.q_stride_h, d.q_stride_q = q.stride(0) * es, q.stride(1) * es, q.stride(2) * es
    d.k, d.v = k.data_ptr(), v.data_ptr()
    d.kv_stride_seg, d.kv_stride_s = k.stride(1) * es, k.stride(2) * es
    d.counts = counts.data_ptr() if counts is not None else None
    d.out = out.data_ptr()
    d.out_stride_b, d.out_stride_h, d.out_stride_q = out.stride(0) * es, out.stride(1) * es, out.stride(2) * es
    d.workspace, d.workspace_bytes = None, 0
    d.status = ops.status_word(q.device).data_ptr()
    d.scale = 1.0 / math.sqrt(D)
    d.dtype = ops._DTYPE_CODE[q.dtype]
    d.batch, d.q_heads, d.kv_heads, d.head_dim, d.q_len, d.num_selected = B, Hq, Hk, D, Q, S
    return d


def _noalloc():
    from mserve_b200._lib import AttnDesc, lib
    fn = lib().mskv_sparse_attention_noalloc
    fn.restype = C.c_int
    fn.argtypes = [C.POINTER(AttnDesc), C.c_void_p]
    return fn


@pytest.mark.parametrize("seed", [0])
def test_noalloc_attention_matches_workspace_entry_point(built_lib, seed):
    from mserve_b200 import ops
    from mserve_b200._lib import check
    fn = _noalloc()
    g = torch.Generator().manual_seed(seed)
    cases = [  # B, Hq, Hkv, Q, S, D, dtype, with counts
        (8, 28, 4, 1, 2176, 128, torch.bfloat16, False),   # the Qwen2.5-VL-7B decode selection
        (3, 16, 2, 1, 700, 64, torch.float16, True),
        (32, 56, 8, 1, 1152, 128, torch.bfloat16, True),   # streaming cluster kernel: no scratch
        (3, 16, 1, 1, 43008, 128, torch.bfloat16, True),   # split path, 3 x 336 splits: 8,386,560 of 8,388,608 bytes
    ]
    from mserve_b200._lib import MSKV_NOALLOC_SCRATCH_BYTES
    for B, Hq, Hkv, Q, S, D, dt, with_counts in cases:
        q = torch.randn(B, Hq, Q, D, generator=g).to(dt).cuda()
        k = torch.randn(B, Hkv, S, D, generator=g).to(dt).cuda()
        v = torch.randn(B, Hkv, S, D, generator=g).to(dt).cuda()
        counts = torch.randint(0, S + 1, (B, Hkv), generator=g, dtype=torch.int32).cuda() if with_counts else None
        ref = ops.sparse_attention(q, k, v, counts=counts)          # existing entry point
        out = torch.full_like(ref, float("nan"))
        stream = torch.cuda.current_stream()
        d = _desc(q, k, v, counts, out)
        from mserve_b200._lib import lib
        assert lib().mskv_attention_workspace_bytes(C.byref(d)) <= MSKV_NOALLOC_SCRATCH_BYTES
        check(fn(C.byref(d), C.c_void_p(stream.cuda_stream)))
        torch.cuda.synchronize()
        ops.check_status(q.device, "noalloc attention")
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), "outputs differ from the workspace entry point"


def test_noalloc_attention_rejects_oversized_shape(built_lib):
    from mserve_b200._lib import MSKV_ERR_RANGE
    fn = _noalloc()
    B, Hq, Hkv, S, D = 3, 16, 1, 43009, 128     # one split more per segment than the widest case above: 8,411,520 bytes
    # every declared row is allocated, so the call could not read past a buffer even if it ran
    q = torch.zeros(B, Hq, 1, D, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(B, Hkv, S, D, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros_like(q)
    d = _desc(q, k, k, None, out)
    assert fn(C.byref(d), C.c_void_p(torch.cuda.current_stream().cuda_stream)) == MSKV_ERR_RANGE
