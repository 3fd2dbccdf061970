"""Generates tests/golden/filter_vectors.npz by running MServe's dual_attention_filter on CPU.

    python tests/golden/make_filter_golden.py [--reference /root/reference]

The reference module (qwen-eljrte/Qwen_Transformer/dual_attention_filter.py, which imports only
torch, math and time) is loaded unmodified from the reference tree and run on seeded attention
probabilities: softmax over keys of N(0, 2^2) logits.  Only the text x image block of batch 0
is stored (the function reads nothing else), together with the arguments, the returned
indices and text_seq, and the block's column sums / maxima as torch computes them.  bf16
blocks are stored as uint16 bit patterns.  Tests never read the reference tree.
"""
from __future__ import annotations

import argparse
import importlib.util
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

CASES = [  # name, dtype, H, v_token_start, img_seq, text_seq, global_thr, individual_thr, use_fp16
    ("thr_small", torch.float32, 4, 15, 300, 40, 0.002, 0.01, False),
    ("heads28", torch.float32, 28, 5, 150, 12, 0.004, 0.02, False),
    ("defaults", torch.float32, 3, 2, 97, 7, 1.0, 0.0, False),
    ("bf16", torch.bfloat16, 4, 8, 200, 24, 0.003, 0.01, False),
    ("fp16_round", torch.float32, 4, 15, 300, 40, 0.002, 0.01, True),
    # the arguments of the reference's call site (attention.py:1331): v_token_start 15,
    # global_thr 0.001, individual_thr 0.01; Qwen2.5-VL-7B's 28 heads, a 14 x 14 token image
    ("callsite", torch.float32, 28, 15, 196, 45, 0.001, 0.01, False),
]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    ap.add_argument("--out", default=str(HERE / "filter_vectors.npz"))
    args = ap.parse_args()
    src = Path(args.reference) / "qwen-eljrte/Qwen_Transformer/dual_attention_filter.py"
    spec = importlib.util.spec_from_file_location("ref_dual_attention_filter", src)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    out = {}
    for n, (name, dtype, H, start, img, text, gthr, ithr, fp16) in enumerate(CASES):
        g = torch.Generator().manual_seed(100 + n)
        T = start + img + text
        # per-key bias shared by every row and head: some tokens are ignored by all of them
        logits = torch.randn(1, H, T, T, generator=g) * 1.5 + torch.randn(T, generator=g) * 2.5
        attn = torch.softmax(logits, dim=-1).to(dtype)
        idx, text_seq = mod.dual_attention_filter(attn, start, img, global_thr=gthr, individual_thr=ithr,
                                                  use_fp16=fp16)
        block = attn[0, :, start + img:start + img + text, start:start + img]
        hm = (block.half() if fp16 and block.dtype == torch.float32 else block).mean(dim=0)
        out[f"{name}/block"] = (block.contiguous().view(torch.int16).numpy().view(np.uint16)
                                if dtype == torch.bfloat16 else block.contiguous().numpy())
        out[f"{name}/meta"] = np.array([H, start, img, text, T, int(fp16), int(dtype == torch.bfloat16)])
        out[f"{name}/thr"] = np.array([gthr, ithr], dtype=np.float64)
        out[f"{name}/idx"] = idx.numpy()
        out[f"{name}/text_seq"] = np.array([text_seq])
        out[f"{name}/attn_sum"] = hm.sum(dim=0).float().numpy()
        out[f"{name}/text_max"] = hm.amax(dim=0).float().numpy()
        print(name, "kept", idx.numel(), "of", img)
    np.savez_compressed(args.out, **out)
    print("wrote", args.out)


if __name__ == "__main__":
    main()
