"""Generates tests/golden/filter_vectors.npz by running MServe's dual_attention_filter on CPU.

    python tests/golden/make_filter_golden.py --reference <MServe checkout>
    (or MSERVE_REFERENCE=<MServe checkout> python tests/golden/make_filter_golden.py)

The reference module (qwen-eljrte/Qwen_Transformer/dual_attention_filter.py, which imports only
torch, math and time) is loaded unmodified from the reference tree and run on seeded attention
probabilities: softmax over keys of N(0, 2^2) logits.  Only the text x image block of batch 0
is stored (the function reads nothing else), together with the arguments, the returned
indices and text_seq, and the block's column sums / maxima as torch computes them.  bf16
blocks are stored as uint16 bit patterns.  Tests never read the reference tree.

The "ithr_*" cases pin the individual threshold's rounding: torch casts the Python scalar to
the block's dtype before `text_max < individual_thr`, so with a threshold that rounds down in
that dtype (bf16(0.001) = 0.00099945..., f16(0.0011) = 0.00109958...) a column whose maximum
equals the rounded threshold is kept.  Three columns are overwritten in every head with a tiny
value and one text row set to the rounded threshold, the next value below it and the next
above it, so their column sums stay far below the global threshold and only the maximum
decides.
"""
from __future__ import annotations

import argparse
import importlib.util
import os
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
    # thresholds that round down in the stage dtype; crafted columns at the threshold
    ("ithr_bf16", torch.bfloat16, 4, 8, 200, 24, 0.003, 0.001, False),
    ("ithr_f16", torch.float16, 4, 8, 200, 24, 0.003, 0.0011, False),
    ("ithr_fp16_mode", torch.float32, 4, 8, 200, 24, 0.003, 0.0011, True),
]
CRAFTED_COLUMNS = (10, 50, 120)


def _stage_dtype(dtype, fp16):
    return torch.float16 if (fp16 or dtype == torch.float16) else dtype


def _neighbours(x: float, sdt: torch.dtype):
    """x rounded to sdt, and the next representable values of sdt below and above it."""
    r = torch.tensor([x], dtype=torch.float32).to(sdt)
    if sdt == torch.float32:
        bits = r.view(torch.int32)
    else:
        bits = r.view(torch.int16)
    below = (bits - 1).view(sdt)
    above = (bits + 1).view(sdt)
    return [float(v) for v in (r, below, above)]


def craft_threshold_columns(attn, start, img, text, ithr, sdt):
    """Columns CRAFTED_COLUMNS of the text x image block: 1e-5 everywhere except text row 3,
    which holds (in every head) the rounded threshold, the value below it and the one above."""
    blk = attn[0, :, start + img:start + img + text, start:start + img]
    for c, v in zip(CRAFTED_COLUMNS, _neighbours(ithr, sdt)):
        blk[:, :, c] = 1e-5
        blk[:, 3, c] = v


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("MSERVE_REFERENCE"),
                    help="root of an MServe checkout (default: $MSERVE_REFERENCE)")
    ap.add_argument("--out", default=str(HERE / "filter_vectors.npz"))
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set MSERVE_REFERENCE to the root of an MServe checkout")
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
        if name.startswith("ithr_"):
            craft_threshold_columns(attn, start, img, text, ithr, _stage_dtype(dtype, fp16))
        idx, text_seq = mod.dual_attention_filter(attn, start, img, global_thr=gthr, individual_thr=ithr,
                                                  use_fp16=fp16)
        block = attn[0, :, start + img:start + img + text, start:start + img]
        hm = (block.half() if fp16 and block.dtype == torch.float32 else block).mean(dim=0)
        out[f"{name}/block"] = (block.contiguous().view(torch.int16).numpy().view(np.uint16)
                                if dtype == torch.bfloat16 else block.contiguous().numpy())
        out[f"{name}/meta"] = np.array([H, start, img, text, T, int(fp16), int(dtype == torch.bfloat16),
                                        int(dtype == torch.float16)])
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
