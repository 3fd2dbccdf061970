"""The two fast paths of mskv_sparse_attention, and the properties the decode engine relies on.

Selections of up to 8 x 4096 rows run one streaming kernel whose CTAs of a (sequence, KV head)
segment form a cluster of ceil(width / 256) <= 8 CTAs; wider ones run the split-sequence
kernels.  Checked here:
  * every cluster size (1..8) and the split path against the oracle (tolerance as in
    test_attention_gpu: 2e-2 of max |out| for 16-bit outputs, the GPU in fp32, the oracle in fp64);
  * outputs of a segment do not depend on the other segments of the call: a batch slice or a
    subset of KV heads gives bit-identical rows (head-sharded ranks and chunked decode steps
    compare bit for bit against the whole layer);
  * rows between a segment's count and the selection width are never read into the result,
    even when they hold NaN;
  * a CUDA-graph replay gives the eager result.
"""
import numpy as np
import pytest
import torch

from oracle import kv_oracle as ko

pytestmark = pytest.mark.gpu


def _close(got: torch.Tensor, ref: np.ndarray, rtol: float):
    g = got.float().cpu().numpy().astype(np.float64)
    scale = np.abs(ref).max() + 1e-30
    err = np.abs(g - ref).max() / scale
    assert err <= rtol, f"max error {err:.3e} (relative to max |out|)"


def _inputs(B, Hq, Hkv, Q, S, D, dtype, seed, with_counts=True):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, Q, D, generator=g).to(dtype)
    k = torch.randn(B, Hkv, S, D, generator=g).to(dtype)
    v = torch.randn(B, Hkv, S, D, generator=g).to(dtype)
    counts = torch.randint(1, S + 1, (B, Hkv), generator=g, dtype=torch.int32) if with_counts else None
    return q, k, v, counts


@pytest.mark.parametrize("S", [1, 200, 300, 700, 1000, 1100, 1300, 1700, 2049])   # clusters of 1, 1, 2, ..., 8
@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float16, 64)])
def test_cluster_sizes_match_oracle(built_lib, S, dtype, D):
    from mserve_b200 import ops
    q, k, v, counts = _inputs(3, 28, 4, 1, S, D, dtype, seed=S)
    out = ops.sparse_attention(q.cuda(), k.cuda(), v.cuda(), counts=counts.cuda())
    torch.cuda.synchronize()
    ops.check_status(out.device, "attention")
    ref = ko.sparse_sdpa_attention(q.double().numpy(), k.double().numpy(), v.double().numpy(), counts=counts.numpy())
    _close(out, ref, 2e-2)


def test_wide_selection_split_path_matches_oracle(built_lib):
    from mserve_b200 import ops
    q, k, v, counts = _inputs(1, 8, 1, 2, 40000, 128, torch.bfloat16, seed=7)
    out = ops.sparse_attention(q.cuda(), k.cuda(), v.cuda(), counts=counts.cuda())
    torch.cuda.synchronize()
    ops.check_status(out.device, "attention")
    ref = ko.sparse_sdpa_attention(q.double().numpy(), k.double().numpy(), v.double().numpy(), counts=counts.numpy())
    _close(out, ref, 2e-2)


def test_segments_are_independent_of_the_call(built_lib):
    """A batch slice and a KV-head subset reproduce the whole call's rows bit for bit."""
    from mserve_b200 import ops
    q, k, v, counts = _inputs(8, 28, 4, 1, 2176, 128, torch.bfloat16, seed=11)
    q, k, v, counts = q.cuda(), k.cuda(), v.cuda(), counts.cuda()
    full = ops.sparse_attention(q, k, v, counts=counts)
    part_b = ops.sparse_attention(q[2:5], k[2:5], v[2:5], counts=counts[2:5].contiguous())
    part_h = ops.sparse_attention(q[:, 7:21].contiguous(), k[:, 1:3].contiguous(), v[:, 1:3].contiguous(),
                                  counts=counts[:, 1:3].contiguous())
    torch.cuda.synchronize()
    ops.check_status(q.device, "attention")
    assert torch.equal(part_b.view(torch.int16), full[2:5].view(torch.int16))
    assert torch.equal(part_h.view(torch.int16), full[:, 7:21].view(torch.int16))


@pytest.mark.parametrize("S", [700, 40000])   # streaming cluster kernel, split path
def test_rows_past_the_count_are_ignored(built_lib, S):
    from mserve_b200 import ops
    q, k, v, counts = _inputs(2, 16, 2, 1, S, 128, torch.bfloat16, seed=S + 1)
    counts[0, 0], counts[1, 1] = S - 5, 17
    kz, vz = k.clone(), v.clone()
    kn, vn = k.clone(), v.clone()
    for b in range(2):
        for h in range(2):
            n = int(counts[b, h])
            kz[b, h, n:], vz[b, h, n:] = 0, 0
            kn[b, h, n:], vn[b, h, n:] = float("nan"), float("nan")
    c = counts.cuda()
    out_z = ops.sparse_attention(q.cuda(), kz.cuda(), vz.cuda(), counts=c)
    out_n = ops.sparse_attention(q.cuda(), kn.cuda(), vn.cuda(), counts=c)
    torch.cuda.synchronize()
    ops.check_status(out_z.device, "attention")
    assert not torch.isnan(out_n.float()).any()
    assert torch.equal(out_n.view(torch.int16), out_z.view(torch.int16))


def test_graph_replay_matches_eager(built_lib):
    from mserve_b200 import ops
    q, k, v, counts = _inputs(8, 28, 4, 1, 2176, 128, torch.bfloat16, seed=5)
    q, k, v, counts = q.cuda(), k.cuda(), v.cuda(), counts.cuda()
    out = torch.empty_like(q)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ops.sparse_attention(q, k, v, counts=counts, out=out)      # warm-up outside the capture
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            ops.sparse_attention(q, k, v, counts=counts, out=out)
    torch.cuda.current_stream().wait_stream(s)
    q.copy_(torch.randn(q.shape, generator=torch.Generator().manual_seed(6)).to(q.dtype).cuda())
    graph.replay()
    torch.cuda.synchronize()
    eager = ops.sparse_attention(q, k, v, counts=counts)
    torch.cuda.synchronize()
    ops.check_status(q.device, "attention")
    assert torch.equal(out.view(torch.int16), eager.view(torch.int16))
    del graph
