"""Parity of the decode attention over selected rows (mskv_sparse_attention) with the oracle.

Tolerance: 2e-2 relative (to the output's magnitude) for bf16/fp16 outputs, 1e-4 for fp32 --
the GPU computes in fp32, the oracle in fp64.
"""
import numpy as np
import pytest
import torch

from conftest import from_bits
from oracle import kv_oracle as ko

pytestmark = pytest.mark.gpu


def _close(got: torch.Tensor, ref: np.ndarray, rtol: float):
    g = got.float().cpu().numpy().astype(np.float64)
    scale = np.abs(ref).max() + 1e-30
    err = np.abs(g - ref).max() / scale
    assert err <= rtol, f"max error {err:.3e} (relative to max |out|)"


@pytest.mark.parametrize("dtype,rtol", [(torch.bfloat16, 2e-2), (torch.float16, 2e-2), (torch.float32, 1e-4)])
@pytest.mark.parametrize("B,Hq,Hkv,Q,S,D", [(8, 28, 4, 1, 2176, 128), (2, 8, 8, 1, 300, 128), (1, 4, 1, 2, 37, 64),
                                            (3, 28, 4, 1, 1, 128), (1, 16, 1, 1, 100, 128), (1, 2, 2, 1, 40, 96)])
def test_sparse_attention(built_lib, dtype, rtol, B, Hq, Hkv, Q, S, D):
    from mserve_b200.selection import sparse_sdpa_attention
    g = torch.Generator().manual_seed(B * 1000 + S)
    q = torch.randn(B, Hq, Q, D, generator=g).to(dtype)
    k = torch.randn(B, Hkv, S, D, generator=g).to(dtype)
    v = torch.randn(B, Hkv, S, D, generator=g).to(dtype)
    out = sparse_sdpa_attention(q.cuda(), None, None, k.cuda(), v.cuda(), None)
    assert out.shape == (B, Hq, Q, D) and out.dtype == dtype
    ref = ko.sparse_sdpa_attention(q.double().numpy(), k.double().numpy(), v.double().numpy())
    _close(out, ref, rtol)


def test_sparse_attention_counts(built_lib):
    from mserve_b200 import ops
    g = torch.Generator().manual_seed(1)
    B, Hq, Hkv, S, D = 3, 28, 4, 700, 128
    q = torch.randn(B, Hq, 1, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, S, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, S, D, generator=g).to(torch.bfloat16)
    counts = torch.randint(0, S + 1, (B, Hkv), generator=g, dtype=torch.int32)
    counts[0, 0] = 0
    counts[1, 1] = 513
    out = ops.sparse_attention(q.cuda(), k.cuda(), v.cuda(), counts=counts.cuda())
    ref = ko.sparse_sdpa_attention(q.double().numpy(), k.double().numpy(), v.double().numpy(), counts=counts.numpy())
    _close(out, ref, 2e-2)
    assert (out[0, :7].float() == 0).all()        # a head with no selected rows outputs zeros


@pytest.mark.parametrize("case,rtol", [("attn_f64", 1e-4), ("attn_bf16", 2e-2), ("attn_f32_q2", 1e-4)])
def test_sparse_attention_reference_golden(built_lib, golden, case, rtol):
    """Against the reference sparse_sdpa_attention's own outputs (repeat_kv'd heads there)."""
    from mserve_b200.selection import sparse_sdpa_attention
    dt = str(golden[f"{case}/dtype"])
    src = torch.bfloat16 if "bfloat16" in dt else torch.float64
    comp = torch.bfloat16 if src == torch.bfloat16 else torch.float32
    q = from_bits(golden[f"{case}/q"], src).to(comp)
    k = from_bits(golden[f"{case}/k_sel"], src).to(comp)
    v = from_bits(golden[f"{case}/v_sel"], src).to(comp)
    ref = from_bits(golden[f"{case}/out"], src).double().numpy()
    out = sparse_sdpa_attention(q.cuda(), None, None, k.cuda(), v.cuda(), None)
    _close(out, ref, rtol)
