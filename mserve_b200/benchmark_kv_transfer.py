"""KV transfer benchmark: selected-row gather host->HBM and row write-back HBM->host.

Rewrite of MServe's benchmark_kv_transfer (qwen-eljrte/benchmark_kv_transfer.py:46-357) for
the B200 library.  Two modes:

``--mode methods`` (the reference's comparison, benchmark_kv_transfer.py:89-177, defaults
B1 H8 T8192 D128 S2048 at lines 27-33): per-token memcpy, CPU index_select + one H2D copy,
and the UVA gather, on the same pinned [B, H, T, D] cache and the same scattered indices
(generate_scattered_indices, lines 59-85, restated).  Unlike the reference the three results
are checked against each other bit for bit, and times come from CUDA events.

``--mode sweep`` (the transfer sweep): one layer in token-major layout [131072 tokens,
8 KV heads, 128] in bf16 and fp8 e4m3 (values ~N(0,1) cast, seed 4); selection density
1/5/10/25/50 %; index structure uniform-random (sorted) vs contiguous runs of 16 and 64
tokens.  For each point it reports the gather GB/s (selected token rows = all heads of a
token, 2 KiB bf16 / 1 KiB fp8, host->HBM) and the write-back GB/s (the same number of rows,
HBM->host ring positions), each against the pinned cudaMemcpyAsync peak of this GPU's host
link in the same direction: one transfer alone (replayed as a CUDA graph: its launch and ramp
on the device included, the host time of the Python call not; that call's own rate is
gather_api_call_gbs), a train of 8 back to back (as a decode loop issues them), and, as the
reference for that transfer size, a pinned cudaMemcpyAsync of the same byte count.  Under torchrun every rank runs the sweep on its own GPU and host
link; rank 0 prints per-point aggregate GB/s (sum over ranks, time = max over ranks) against the
aggregate memcpy peak (every rank's peak measured at the same time, summed).

Prints one JSON object per line.
"""
from __future__ import annotations

import argparse
import json
import os
import time
from typing import List

import numpy as np
import torch

from . import cuda_uva, ops


# ------------------------------------------------------------------------------- shared pieces
def generate_scattered_indices(seq_len: int, num_selected: int, seed: int = 42) -> torch.Tensor:
    """Scattered unique indices with a minimum gap where possible, in shuffled order.

    Restates generate_scattered_indices (qwen-eljrte/benchmark_kv_transfer.py:59-85): the
    same random calls in the same order, so a given seed yields the reference's indices."""
    torch.manual_seed(seed)
    np.random.seed(seed)
    indices: List[int] = []
    min_gap = seq_len // (num_selected * 2)
    attempts = 0
    while len(indices) < num_selected and attempts < num_selected * 10:
        idx = np.random.randint(0, seq_len)
        if all(abs(idx - e) >= min_gap for e in indices):
            indices.append(idx)
        attempts += 1
    while len(indices) < num_selected:
        idx = np.random.randint(0, seq_len)
        if idx not in indices:
            indices.append(idx)
    t = torch.tensor(indices, dtype=torch.long)
    return t[torch.randperm(len(t))]


def structured_indices(n_tokens: int, n_sel: int, run: int, gen: torch.Generator) -> torch.Tensor:
    """Sorted unique token indices: uniform random (run = 1) or contiguous runs of `run`."""
    if run <= 1:
        return torch.randperm(n_tokens, generator=gen)[:n_sel].sort().values
    n_runs = max(1, n_sel // run)
    starts = torch.randperm(n_tokens // run, generator=gen)[:n_runs].sort().values * run
    idx = (starts[:, None] + torch.arange(run)[None, :]).reshape(-1)
    return idx[:n_sel].sort().values


TRAIN = 8   # gathers per back-to-back train


def graph_timed(fn, reps: int) -> float:
    """Median milliseconds of fn() captured as a CUDA graph and replayed alone (the device time of
    its kernels, without the host time of the Python call)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        fn()
    ms = timed(g.replay, reps)
    del g
    return ms


def timed(fn, reps: int, warmup: int = 2) -> float:
    """Median milliseconds of fn() over reps, CUDA events on the current stream."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        ts.append(e0.elapsed_time(e1))
    ts.sort()
    return ts[len(ts) // 2]


def memcpy_peaks(device: torch.device, nbytes: int = 256 << 20, reps: int = 5) -> dict:
    h = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    g = torch.empty(nbytes, dtype=torch.uint8, device=device)
    h2d = nbytes / (timed(lambda: g.copy_(h, non_blocking=True), reps) * 1e-3) / 1e9
    d2h = nbytes / (timed(lambda: h.copy_(g, non_blocking=True), reps) * 1e-3) / 1e9
    return {"h2d": h2d, "d2h": d2h}


# ------------------------------------------------------------------------------- methods mode
def run_methods(args, device) -> dict:
    B, H, T, D, S = args.batch_size, args.num_heads, args.seq_len, args.head_dim, args.num_selected
    g = torch.Generator().manual_seed(0)
    k = torch.randn(B, H, T, D, generator=g).to(torch.bfloat16).pin_memory()
    v = torch.randn(B, H, T, D, generator=g).to(torch.bfloat16).pin_memory()
    idx = generate_scattered_indices(T, S)
    nbytes = 2 * B * H * S * D * 2
    out = {"mode": "methods", "config": {"B": B, "H": H, "T": T, "D": D, "S": S}, "bytes": nbytes}

    kd = torch.empty(B, H, S, D, dtype=torch.bfloat16, device=device)
    vd = torch.empty_like(kd)

    def per_token():                       # method 1 (benchmark_kv_transfer.py:89-114)
        for i, t in enumerate(idx.tolist()):
            kd[:, :, i, :].copy_(k[:, :, t, :], non_blocking=True)
            vd[:, :, i, :].copy_(v[:, :, t, :], non_blocking=True)
    kp = torch.empty(B, H, S, D, dtype=torch.bfloat16).pin_memory()
    vp = torch.empty_like(kp).pin_memory()

    def gather_memcpy():                   # method 2 (benchmark_kv_transfer.py:118-145)
        torch.index_select(k, 2, idx, out=kp)
        torch.index_select(v, 2, idx, out=vp)
        kd.copy_(kp, non_blocking=True)
        vd.copy_(vp, non_blocking=True)
    res = {}

    def uva():                             # method 3 (benchmark_kv_transfer.py:149-177)
        res["k"], res["v"] = cuda_uva.uva_gather(k, v, idx, B, H, T, D)

    results = {}
    for name, fn, reps in (("scattered_memcpy", per_token, max(1, args.iterations // 10)),
                           ("gather_memcpy", gather_memcpy, args.iterations),
                           ("cuda_uva", uva, args.iterations)):
        ms = timed(fn, reps, warmup=min(args.warmup, 3))
        results[name] = {"ms": ms, "GB/s": nbytes / (ms * 1e-3) / 1e9}
        if name == "scattered_memcpy":
            ref_k, ref_v = kd.clone(), vd.clone()
        elif name == "gather_memcpy":
            assert torch.equal(kd, ref_k) and torch.equal(vd, ref_v), "method 2 differs from method 1"
    assert torch.equal(res["k"], ref_k) and torch.equal(res["v"], ref_v), "UVA gather differs from method 1"
    base = results["gather_memcpy"]["ms"]
    for r in results.values():
        r["speedup_vs_gather_memcpy"] = base / r["ms"]
    out["results"] = results
    out["bit_exact"] = True
    out["memcpy_peak_gbs"] = memcpy_peaks(device)
    return out


# ------------------------------------------------------------------------------- sweep mode
def run_sweep(args, device, world: int, rank: int):
    T, H, D = args.sweep_tokens, 8, 128
    # Every rank measures its memcpy peak at the same time; the sum over ranks is the host's
    # aggregate link peak with all GPUs pulling at once, the denominator of the aggregate rate.
    _barrier(world)
    own = memcpy_peaks(device)
    peaks = {"h2d": _sum(own["h2d"], world), "d2h": _sum(own["d2h"], world), "per_rank_h2d": own["h2d"],
             "per_rank_d2h": own["d2h"], "ranks": world}
    gen = torch.Generator().manual_seed(4)
    lines = []
    mc_host = torch.empty(T * H * D * 2 // 2, dtype=torch.uint8).pin_memory()   # the largest point (50%, bf16)
    mc_dev = torch.empty_like(mc_host, device=device)
    for dtype in (torch.bfloat16, torch.float8_e4m3fn):
        es = torch.empty((), dtype=dtype).element_size()
        host = ops.host_empty((T, H, D), dtype)
        vals = torch.randn(T, H, D, generator=gen)
        host.copy_(vals.to(dtype))
        row_bytes = H * D * es
        # token-major layer as one segment whose rows are whole tokens (all heads)
        host_rows = host.view(1, 1, T, H * D)
        for density in (0.01, 0.05, 0.10, 0.25, 0.50):
            for run in (1, 16, 64):
                idx = structured_indices(T, int(T * density), run, gen).to(torch.int32).to(device)
                n_sel = idx.numel()
                dev_rows = torch.empty(1, 1, n_sel, H * D, dtype=dtype, device=device)
                src = ops.strided_rows(host_rows, None, device=device)
                ms_api = timed(lambda: ops.gather(src, idx, dev_rows, None, batch=1), args.iterations)
                ms_g = graph_timed(lambda: ops.gather(src, idx, dev_rows, None, batch=1), args.iterations)
                # a train of TRAIN gathers back to back (as a decode loop issues them): the launch
                # and ramp of one transfer overlap the tail of the previous one
                ms_gt = timed(lambda: [ops.gather(src, idx, dev_rows, None, batch=1) for _ in range(TRAIN)],
                              max(2, args.iterations // 2)) / TRAIN
                # correctness: bit-exact against the host rows
                got = dev_rows.view(torch.uint8).cpu() if es == 1 else dev_rows.view(torch.int16).cpu()
                ref = host_rows[0, 0][idx.cpu().long()]
                ref = ref.view(torch.uint8) if es == 1 else ref.view(torch.int16)
                assert torch.equal(got[0, 0], ref), "gather mismatch"
                # write-back: the same number of rows HBM -> host ring slots
                ring = torch.tensor([int(T // 3)], dtype=torch.int32, device=device)
                dst = ops.strided_rows(host_rows, None, len_scalar=T, ring_start=ring, ring_cap=T, device=device)
                srcw = ops.strided_rows(dev_rows, None, device=device)
                ms_w = graph_timed(lambda: ops.copy_rows(srcw, dst, batch=1, num_tokens=n_sel, device=device),
                                   args.iterations)
                ms_wt = timed(lambda: [ops.copy_rows(srcw, dst, batch=1, num_tokens=n_sel, device=device)
                                       for _ in range(TRAIN)], max(2, args.iterations // 2)) / TRAIN
                ops.check_status(device, "transfer sweep")
                nbytes = n_sel * row_bytes
                # a pinned cudaMemcpyAsync of the same byte count: what the copy engine reaches at
                # this transfer size (contiguous, so an upper reference for a scattered gather)
                ms_mc = timed(lambda: mc_dev[:nbytes].copy_(mc_host[:nbytes], non_blocking=True), args.iterations)
                ms_g, ms_gt, ms_w, ms_wt, ms_mc, ms_api = (_max(x, world) for x in (ms_g, ms_gt, ms_w, ms_wt, ms_mc,
                                                                                   ms_api))
                agg = nbytes * world            # every rank moved nbytes; time = the slowest rank
                line = {"mode": "sweep", "dtype": str(dtype).replace("torch.", ""), "tokens": T, "heads": H,
                        "head_dim": D, "density": density, "structure": "random" if run == 1 else f"runs{run}",
                        "rows": n_sel, "row_bytes": row_bytes, "n_gpus": world,
                        "gather_gbs": agg / (ms_g * 1e-3) / 1e9, "gather_frac_h2d_peak": agg / (ms_g * 1e-3) / 1e9 / peaks["h2d"],
                        "writeback_gbs": agg / (ms_w * 1e-3) / 1e9, "writeback_frac_d2h_peak": agg / (ms_w * 1e-3) / 1e9 / peaks["d2h"],
                        "gather_api_call_gbs": agg / (ms_api * 1e-3) / 1e9,
                        "gather_train_gbs": agg / (ms_gt * 1e-3) / 1e9,
                        "gather_train_frac_h2d_peak": agg / (ms_gt * 1e-3) / 1e9 / peaks["h2d"],
                        "writeback_train_gbs": agg / (ms_wt * 1e-3) / 1e9,
                        "writeback_train_frac_d2h_peak": agg / (ms_wt * 1e-3) / 1e9 / peaks["d2h"],
                        "memcpy_same_bytes_gbs": agg / (ms_mc * 1e-3) / 1e9,
                        "gather_frac_same_bytes_memcpy": ms_mc / ms_g,
                        "gather_ms": ms_g, "writeback_ms": ms_w, "memcpy_peak_gbs": peaks, "bit_exact": True}
                lines.append(line)
                if rank == 0:
                    print(json.dumps(line), flush=True)
    return lines


def _barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def _sum(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def _max(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main():
    ap = argparse.ArgumentParser(description="KV transfer benchmark (B200)")
    ap.add_argument("--mode", choices=["methods", "sweep"], default="methods")
    ap.add_argument("--batch-size", type=int, default=1)
    ap.add_argument("--num-heads", type=int, default=8)
    ap.add_argument("--seq-len", type=int, default=8192)
    ap.add_argument("--head-dim", type=int, default=128)
    ap.add_argument("--num-selected", type=int, default=2048)
    ap.add_argument("--iterations", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--sweep-tokens", type=int, default=131072)
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    try:
        if args.mode == "methods":
            if rank == 0:
                print(json.dumps(run_methods(args, device)), flush=True)
        else:
            run_sweep(args, device, world, rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
