"""The reference's decode-time selection path, timed on the GPU -- baseline infrastructure.

Restates, step for step, one layer of the reference's sparse decode branch
(qwen-eljrte/Qwen_Transformer/attention.py:1942-1997) on one B200, with the reference's own
UVA gather kernel (qwen-eljrte/cuda_uva_kernel.cpp built unmodified by oracle/build_ref.py)
and torch for the rest, exactly as the reference calls it:

  1. get_async (kv_cache.py:241-294): the whole layer's host K and V -- stored with repeat_kv'd
     query heads (attention.py:1930-1934) -- copied host->device into reusable buffers;
  2. get_full_kv (kv_cache.py:631-643): cat(past, new token) on the device;
  3. compute_token_importance (attention.py:532-588): q_last . K^T over all query heads, mean
     over heads, torch.topk, .cpu();
  4. get_sparse_async_uva (kv_cache.py:493-543): torch.cuda.synchronize(), then the reference
     kernel gathers the selected rows of every query head from host memory;
  5. sparse_sdpa_attention (attention.py:591-641): softmax(q K_sel^T / sqrt(D)) V_sel.

The reference selects one index set per sequence and only for batch 1 (its .squeeze(0)), so a
layer is timed per sequence.  The selection size is set to the decode bench's 2176 tokens
(top_k_ratio = 2176/16384) so that both paths select the same number of tokens.  One
deviation, for safety: the index list is pinned before the gather (the reference passes a
pageable CPU tensor, which its kernel dereferences on the device).  Shapes: Qwen2.5-VL-7B,
28 query / 4 KV heads, head_dim 128, 16384 cached tokens, bf16.

    python -m oracle.time_reference_path [--layers 4]
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import math

import torch

from oracle import build_ref


def _same_address_on_device(t: torch.Tensor) -> bool:
    from mserve_b200 import _lib
    p = C.c_void_p()
    rc = _lib.lib().mskv_device_view(C.c_void_p(t.data_ptr()), C.byref(p))
    return rc == _lib.MSKV_OK and p.value == t.data_ptr()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args()
    ref = build_ref.load()
    if ref is None:
        print(json.dumps({"unavailable": "oracle/_ref/cuda_uva_ref.so is not built"}))
        return
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    Hq, Hkv, D, T, S = 28, 4, 128, 16384, 2176
    G = Hq // Hkv
    ratio, min_tokens = S / T, 128
    g = torch.Generator().manual_seed(0)
    layers = []
    for _ in range(args.layers):                  # host caches as the reference stores them
        k = torch.randn(1, Hkv, T, D, generator=g).to(torch.bfloat16)
        v = torch.randn(1, Hkv, T, D, generator=g).to(torch.bfloat16)
        k_rep = k[:, :, None].expand(1, Hkv, G, T, D).reshape(1, Hq, T, D).contiguous().pin_memory()
        v_rep = v[:, :, None].expand(1, Hkv, G, T, D).reshape(1, Hq, T, D).contiguous().pin_memory()
        if not (_same_address_on_device(k_rep) and _same_address_on_device(v_rep)):
            print(json.dumps({"unavailable": "pinned memory not device-accessible at its host address"}))
            return
        layers.append((k_rep, v_rep))
    kbuf = torch.empty(1, Hq, T, D, dtype=torch.bfloat16, device=dev)
    vbuf = torch.empty_like(kbuf)
    h2d = torch.cuda.Stream(dev)
    q = torch.randn(1, Hq, 1, D, generator=g).to(torch.bfloat16).to(dev)
    k_new = torch.randn(1, Hq, 1, D, generator=g).to(torch.bfloat16).to(dev)
    v_new = torch.randn(1, Hq, 1, D, generator=g).to(torch.bfloat16).to(dev)

    def layer_step(k_host, v_host, parts):
        cur = torch.cuda.current_stream(dev)
        e = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
        e[0].record(cur)
        with torch.cuda.stream(h2d):                               # 1. get_async
            h2d.wait_stream(cur)
            kbuf.copy_(k_host, non_blocking=True)
            vbuf.copy_(v_host, non_blocking=True)
            done = torch.cuda.Event()
            done.record(h2d)
        cur.wait_event(done)
        e[1].record(cur)
        key_full = torch.cat([kbuf, k_new], dim=2)                 # 2. get_full_kv
        value_full = torch.cat([vbuf, v_new], dim=2)
        e[2].record(cur)
        scores = torch.matmul(q[:, :, -1:, :], key_full.transpose(-1, -2)).squeeze(2)   # 3. importance
        scores = scores.mean(dim=1)
        k_sel = min(max(min_tokens, int(key_full.shape[2] * ratio)), key_full.shape[2])
        idx = torch.topk(scores, k_sel, dim=-1, sorted=False).indices.squeeze(0).cpu()
        idx = idx[idx < T]                                         # the cached tokens only
        e[3].record(cur)
        torch.cuda.synchronize(dev)                                # 4. get_sparse_async_uva
        idx = idx.pin_memory()
        ks, vs = ref.uva_gather(k_host, v_host, idx, 1, Hq, T, D)
        torch.cuda.synchronize(dev)
        e[4].record(cur)
        att = torch.matmul(q, ks.transpose(-1, -2)) / math.sqrt(D)   # 5. sparse_sdpa_attention
        out = torch.matmul(torch.softmax(att, dim=-1), vs)
        e[5].record(cur)
        e[5].synchronize()
        parts.append([e[i].elapsed_time(e[i + 1]) for i in range(5)] + [e[0].elapsed_time(e[5]), int(idx.numel())])
        return out

    for kh, vh in layers:                                          # warm-up
        layer_step(kh, vh, [])
    parts = []
    for _ in range(args.reps):
        for kh, vh in layers:
            layer_step(kh, vh, parts)
    med = [sorted(p[i] for p in parts)[len(parts) // 2] for i in range(6)]
    layer_bytes = 2 * Hq * T * D * 2
    gather_bytes = 2 * Hq * parts[-1][6] * D * 2
    print(json.dumps({
        "path": "reference decode branch per sequence and layer (attention.py:1942-1997), restated in torch "
                "with the reference's own UVA gather kernel",
        "shape": f"1 sequence x {T} tokens, {Hq}q/{Hkv}kv heads (host cache holds {Hq} repeat_kv'd heads), "
                 f"D {D}, bf16, {S} selected tokens",
        "ms_per_sequence_layer": med[5],
        "ms_parts": {"full_layer_h2d": med[0], "get_full_kv_cat": med[1], "importance_topk_cpu": med[2],
                     "sync_uva_gather_sync": med[3], "sparse_attention": med[4]},
        "bytes": {"full_layer_h2d": layer_bytes, "uva_gather": gather_bytes},
        "gather_gbs": gather_bytes / (med[3] * 1e-3) / 1e9,
        "timing": "CUDA events on the current stream around each step (idle time of the host "
                  "synchronisations included); median over layers x repetitions"}))


if __name__ == "__main__":
    main()
