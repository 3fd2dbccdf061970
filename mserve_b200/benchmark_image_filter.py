"""Timing of the prefill image-token filter (mskv_image_filter) against the reference's torch code.

The reference filters image tokens at prefill with dual_attention_filter
(qwen-eljrte/Qwen_Transformer/dual_attention_filter.py:6-103), called on the fp32 attention
probabilities of eager prefill attention (attention.py:663-681) as
dual_attention_filter(attn_prob, 15, image_token_num, 0.001, 0.01) (attention.py:1331).
Workloads: Qwen2.5-VL-7B's 28 heads, 15 system tokens, an image of 1296 tokens (36 x 36) or
4096 tokens (64 x 64), then 64 / 256 text tokens; fp32 [1, 28, T, T] maps of softmaxed seeded
logits.

Arms, each on the same map and checked to keep the same tokens:
  * mserve: selection.dual_attention_filter (a counter reset and one kernel, then the read of
    the kept count);
  * reference: the reference function's torch operations on the GPU, as it runs them (head
    mean, column sum and max, the two thresholds, the boolean index).
Per arm: the call's wall time up to the kept indices being usable on the host side (a device
synchronisation inside, as both arms have one), median over repetitions, with L2 flushed
(a 256 MB write) before each call.  For mserve also the device time of one call (the counter
reset and the kernel): a CUDA graph of 20 x (L2 flush, call) minus a graph of 20 x flush,
median over replays, divided by 20; and the HBM roofline: algorithmic bytes = heads x text x
image x 4 (the block read) over that time.

    python -m mserve_b200.benchmark_image_filter [--reps 30] [--graph-calls 20] [--only NAME]
"""
from __future__ import annotations

import argparse
import json
import time
from pathlib import Path

import torch

from . import ops
from .selection import dual_attention_filter

WORKLOADS = [  # name, heads, v_token_start, image tokens, text tokens
    ("7b_img1296_text64", 28, 15, 1296, 64),
    ("7b_img4096_text256", 28, 15, 4096, 256),
]
GLOBAL_THR, INDIVIDUAL_THR = 0.001, 0.01


def reference_filter(attn, v_token_start, img_seq, global_thr, individual_thr):
    """The reference function's tensor operations (dual_attention_filter.py:37-70), in torch."""
    B, H, T, _ = attn.shape
    text_seq = T - img_seq - v_token_start
    img_beg, img_end = v_token_start, v_token_start + img_seq
    block = attn[0, :, img_end:img_end + text_seq, img_beg:img_end]
    head_mean = block.mean(dim=0)
    attn_sum = torch.sum(head_mean, dim=0)
    text_max = torch.amax(head_mean, dim=0)
    candidate = (attn_sum < attn_sum.sum() * global_thr) & (text_max < individual_thr)
    return torch.arange(img_seq, device=attn.device)[~candidate].to(torch.long), int(text_seq)


def hbm_peak_gbs():
    p = Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def graph_time_us(fn, flush, calls, reps=7):
    """Device time of one fn() call after an L2 flush: a CUDA graph of `calls` x (flush, fn)
    minus a graph of `calls` x flush, median over replays, divided by `calls`."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):                   # warm-up outside capture
        fn()
    torch.cuda.current_stream().wait_stream(side)
    graphs = []
    for with_fn in (True, False):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(calls):
                flush.zero_()
                if with_fn:
                    fn()
        graphs.append(g)
    times = []
    for g in graphs:
        ts = []
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            e1.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e3)
        times.append(sorted(ts)[reps // 2])
    del graphs
    return (times[0] - times[1]) / calls


def probabilities(H, T, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    logits = torch.randn(1, H, T, T, generator=g, device=dev) * 1.5
    logits += torch.randn(T, generator=g, device=dev) * 2.5
    return torch.softmax(logits, dim=-1)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reps", type=int, default=30)
    ap.add_argument("--graph-calls", type=int, default=20)
    ap.add_argument("--only", choices=[w[0] for w in WORKLOADS], default=None, help="run one workload")
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    peak, peak_kind = hbm_peak_gbs()
    for name, H, start, img, text in WORKLOADS:
        if args.only and name != args.only:
            continue
        T = start + img + text
        attn = probabilities(H, T, seed=img + text, dev=dev)
        ours, ts = dual_attention_filter(attn, start, img, GLOBAL_THR, INDIVIDUAL_THR)
        ref, ts_ref = reference_filter(attn, start, img, GLOBAL_THR, INDIVIDUAL_THR)
        same = torch.equal(ours, ref) and ts == ts_ref

        def wall(fn):
            out = []
            for _ in range(args.reps + 3):
                flush.zero_()
                torch.cuda.synchronize(dev)
                t0 = time.perf_counter()
                idx, _ = fn(attn, start, img, GLOBAL_THR, INDIVIDUAL_THR)
                idx.numel()
                torch.cuda.synchronize(dev)
                out.append(time.perf_counter() - t0)
            out = sorted(out[3:])
            return out[len(out) // 2] * 1e6

        a0 = attn[0]

        def run_filter():
            ops.image_filter(a0, img_start=start, img_seq=img, text_start=start + img, text_seq=text,
                             global_thr=GLOBAL_THR, individual_thr=INDIVIDUAL_THR)

        dev_us = graph_time_us(run_filter, flush, args.graph_calls)
        block_bytes = H * text * img * 4
        achieved = block_bytes / (dev_us * 1e-6) / 1e9
        print(json.dumps({
            "workload": name, "heads": H, "v_token_start": start, "image_tokens": img, "text_tokens": text,
            "attn_map": f"fp32 [1, {H}, {T}, {T}]", "kept": int(ours.numel()), "same_as_reference": bool(same),
            "mserve_call_us": wall(dual_attention_filter), "reference_call_us": wall(reference_filter),
            "mserve_kernels_us": dev_us, "block_bytes": block_bytes,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind},
            "timing": "call times: median over repetitions, L2 flushed before each call; kernel time: CUDA graph of (flush, call) x N minus (flush) x N, over N"}), flush=True)
        del attn


if __name__ == "__main__":
    main()
