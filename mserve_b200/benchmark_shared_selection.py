"""Timing of the head-sharded shared selection (mserve_b200.parallel.SharedSelection).

The selection the reference makes (one index set per sequence from the mean over all query
heads, qwen-eljrte/Qwen_Transformer/attention.py:558-572) with the KV heads sharded over the
ranks of one node: each rank scores its own heads, one NCCL all-gather over NVLink brings every
rank's fp32 score rows to every rank, and the top-k kernel sums them in global head order.

Shape: the Qwen2.5-VL-32B decode shape, 16 sequences x 32768 tokens, 40 query / 8 KV heads,
head_dim 128, bf16 keys in HBM (seed 2), top-4096 + the last 256 tokens per sequence.

    python -m torch.distributed.run --nproc-per-node N -m mserve_b200.benchmark_shared_selection [--exchange peer]

Prints one JSON line on rank 0: per phase (scores, exchange, top-k, whole selection) the
median over repetitions of the CUDA-event time, max over ranks, and the exchanged bytes.
With --exchange peer the score kernel stores the rows into every rank's buffer itself
(parallel.PeerExchange): "scores_us" then covers the scores, their transfer and the flag
waits, and "exchange_us" is zero.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

from . import ops, parallel


def _max(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--tokens", type=int, default=32768)
    ap.add_argument("--exchange", choices=["nccl", "peer"], default="nccl")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        B, Hq, Hkv, D, T, K, R = args.batch, 40, 8, 128, args.tokens, 4096, 256
        sel = parallel.SharedSelection(B, Hkv, Hq, T, device=dev, exchange=args.exchange)
        g = torch.Generator(device=dev).manual_seed(2 + rank)
        k_local = torch.randn(B, sel.Hl, T, D, generator=g, device=dev).to(torch.bfloat16)
        q0, q1 = sel.q_heads_local()
        q_local = torch.randn(B, q1 - q0, D, generator=g, device=dev).to(torch.bfloat16)
        rows = ops.strided_rows(k_local, None, device=dev)
        idx = torch.empty(B, K + R, dtype=torch.int32, device=dev)
        cnt = torch.empty(B, dtype=torch.int32, device=dev)
        scale = 1.0 / Hq

        def phases():
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
            ev[0].record()
            if sel.peer is not None:
                gathered = sel.peer.score(q_local, rows, max_tokens=T)
                ev[1].record()
            else:
                ops.score(q_local, rows, batch=B, kv_heads=sel.Hl, max_tokens=T, out=sel.local)
                ev[1].record()
                gathered = parallel.exchange_head_scores(sel.local, sel.gathered, sel.group)
            ev[2].record()
            ops.topk(gathered, top_k=K, recent=R, len_scalar=T, rows_per_sel=Hkv, sel_per_batch=1,
                     scale=scale, out=idx, counts=cnt, row_blocks=(world, B, sel.Hl))
            ev[3].record()
            return ev

        for _ in range(5):
            phases()
        torch.cuda.synchronize()
        samples = []
        for _ in range(args.reps):
            ev = phases()
            ev[3].synchronize()
            samples.append([ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2]), ev[2].elapsed_time(ev[3]),
                            ev[0].elapsed_time(ev[3])])
        med = [sorted(s[i] for s in samples)[len(samples) // 2] for i in range(4)]
        med = [_max(x, world) for x in med]
        ops.check_status(dev, "shared selection")
        key_bytes = B * sel.Hl * T * D * 2
        xbytes = (world - 1) * B * sel.Hl * T * 4            # score rows received per rank
        if rank == 0:
            print(json.dumps({
                "shape": f"{B} seqs x {T} tokens, {Hq}q/{Hkv}kv heads, D {D}, top-{K} + last {R} per sequence",
                "ranks": world, "kv_heads_per_rank": sel.Hl, "exchange": args.exchange,
                "scores_us": med[0] * 1e3, "exchange_us": med[1] * 1e3, "topk_us": med[2] * 1e3,
                "selection_us": med[3] * 1e3,
                "key_bytes_per_rank": key_bytes, "score_gbs_per_rank": key_bytes / (med[0] * 1e-3) / 1e9,
                "exchange_bytes_received_per_rank": xbytes,
                "exchange_gbs_per_rank": (xbytes / (med[1] * 1e-3) / 1e9) if world > 1 else None,
                "timing": "median of CUDA-event times per phase over repetitions, max over ranks"}), flush=True)
        sel.close()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
