"""Decode-step benchmark of the B200 KV selection-and-offload path.

Workload (Qwen2.5-VL-7B decode selection): 28 layers, 28 query / 4 KV heads, head_dim 128,
bf16; 8 sequences of 16384 tokens (first 75% ~N(0,1) "image" KV, rest ~N(0,0.5)); all K and V
in pinned host memory, K also in HBM key pages for scoring; q ~N(0,1).  One step = one decode
step over all 28 layers: GQA-summed scores -> top-2048 of the non-window tokens ∪ the last 128
per (sequence, KV head) -> UVA gather of the selected K/V rows from host memory into HBM ->
attention over them.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mserve|reference] [--workload W]

N ranks (torchrun, one per GPU) split this one problem: the KV heads first, then the sequences
when there are more ranks than KV heads (mserve_b200.parallel.shard_plan), each sequence group
taking sequences in proportion to the slowest concurrent host-link rate among its ranks, measured
at start-up (evenly when the links are equally fast); parallel.plan_for_links groups the KV heads
more coarsely instead when the measured rates make that more than 3% faster.  Every rank holds its
(sequence, KV head) pairs in its own host store and gathers them over its own host link; there
is no collective on the data path ("scaling": "strong": the total work is fixed).  The KV and
queries of every (layer, sequence, head) come from their own seed, so each N computes exactly the
same numbers, and every rank checks bit for bit that its share equals the unsharded layer
computed on its GPU (the line's "parity").  The line's "shared_selection" field times the
reference's head-averaged selection with the heads on the ranks: the NCCL all-gather of score
rows, and the score kernel's own stores into the peers' buffers (exchange="peer").

Prints one JSON line (rank 0).  value = selected K+V bytes gathered host->HBM per second over
the whole step (all ranks), ms_per_step = decode-step time (max over ranks).  --impl reference
times the C restatement of the reference's CPU path (oracle/oracle_kv.c: scores, selection,
index_select gather + the H2D copy of the gathered rows, attention) on all 28 layers on the
host cores, rank 0 only.  The line's decode_loop field times the same step in a decode loop
that appends each step's token to every layer (begin_step() and a step captured with
k_new/v_new), so the cache grows as the loop runs.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import socket
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "selected-KV gather GB/s host→HBM vs PCIe peak; decode step ms at 1/2/4/8 B200"
# The decode-selection workloads.  image_frac: the first fraction of every sequence's KV is
# ~N(0,1) ("image" tokens), the rest ~N(0,0.5) ("text").
WORKLOADS = {
    "qwen7b": (dict(layers=28, batch=8, q_heads=28, kv_heads=4, head_dim=128, seq_len=16384, top_k=2048,
                    recent=128, image_frac=0.75, seed=0),
               "qwen2.5-vl-7b decode selection: 28 layers, 28q/4kv heads, head_dim 128, bf16, 8 seqs x 16384 "
               "tokens, top-2048 + last-128 per (seq, kv head), KV in pinned host"),
    "qwen32b": (dict(layers=64, batch=16, q_heads=40, kv_heads=8, head_dim=128, seq_len=32768, top_k=4096,
                     recent=256, image_frac=1.0, seed=2),
                "qwen2.5-vl-32b decode selection: 64 layers, 40q/8kv heads, head_dim 128, bf16, 16 seqs x 32768 "
                "tokens, KV ~N(0,1), top-4096 + last-256 per (seq, kv head), KV in pinned host"),
    # multi-turn: context lengths uniform in [4096, 65536] (seed 3); one timed turn appends 2880
    # image + 64 text tokens per sequence (16-token HBM key pages + host write-through), then
    # decode selects the top ceil(10% of L_b) tokens per (sequence, KV head)
    "llava34b": (dict(layers=60, batch=32, q_heads=56, kv_heads=8, head_dim=128, seq_len=65536, top_k=0,
                      top_k_ratio=0.1, recent=0, image_frac=1.0, lens_uniform=(4096, 65536), lens_seed=3,
                      turn_image=2880, turn_text=64, seed=3),
                 "llava-v1.6-34b multi-turn decode selection: 60 layers, 56q/8kv heads, head_dim 128, bf16, 32 seqs "
                 "with contexts uniform in [4096, 65536], a 2880 image + 64 text token append turn, then top-10% "
                 "per (seq, kv head), KV in pinned host"),
}
# The sizes the link-peak copies use (a copy of 1 GiB runs ~20 ms: start skew between ranks is
# negligible against it).
PEAK_BYTES = 1 << 30
PEAK_REPS = 5


def workload_lens(wl):
    """Context length of every sequence of the workload."""
    if "lens_uniform" in wl:
        lo, hi = wl["lens_uniform"]
        rng = np.random.default_rng(wl["lens_seed"])
        return [int(x) for x in rng.integers(lo, hi, size=wl["batch"], endpoint=True)]
    return [wl["seq_len"]] * wl["batch"]


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["mserve", "reference"], default="mserve")
    ap.add_argument("--layers", type=int, default=None, help="override the layer count (smaller test runs only)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-decode-loop", action="store_true")
    ap.add_argument("--no-exchange", action="store_true", help="skip the shared-selection exchange timing")
    ap.add_argument("--no-parity", action="store_true", help="skip the per-rank check against the unsharded layer")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the 32B-shape decode (4 layers), the 34B multi-turn decode (2 layers) and the "
                         "transfer-sweep points of the line")
    ap.add_argument("--chunks", type=int, default=4, help="sequence chunks pipelined per layer")
    ap.add_argument("--gather-ctas", type=int, default=0,
                    help="CTAs of each host-memory gather (0: the library's default bound)")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="qwen7b",
                    help="qwen7b (the headline workload), qwen32b (64 layers need ~140 GB of pinned host memory "
                         "in all: use --layers on smaller hosts) or llava34b")
    return ap.parse_args()


# ------------------------------------------------------------------------------------- helpers
def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def _reduce(x: float, world: int, op) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=op)
    return float(t.item())


def max_over_ranks(x: float, world: int) -> float:
    import torch.distributed as dist
    return _reduce(x, world, dist.ReduceOp.MAX if world > 1 else None)


def min_over_ranks(x: float, world: int) -> float:
    import torch.distributed as dist
    return _reduce(x, world, dist.ReduceOp.MIN if world > 1 else None)


def sum_over_ranks(x: float, world: int) -> float:
    import torch.distributed as dist
    return _reduce(x, world, dist.ReduceOp.SUM if world > 1 else None)


def gather_objects(obj, world: int):
    if world == 1:
        return [obj]
    import torch.distributed as dist
    out = [None] * world
    dist.all_gather_object(out, obj)
    return out


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None

    def __enter__(self):
        """Starts sampling every 50 ms and returns once the first sample is in (at most 3 s), so
        the samples cover the work that follows."""
        self.lines = []
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.idx), "-lms", "50"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return self
        import selectors
        sel = selectors.DefaultSelector()
        sel.register(self.proc.stdout, selectors.EVENT_READ)
        if sel.select(timeout=3.0):
            first = self.proc.stdout.readline()
            if first.strip():
                self.lines.append(first)
        sel.close()
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines += [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            p = [x.strip() for x in l.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def pcie_peaks(device, world, nbytes=PEAK_BYTES, reps=PEAK_REPS):
    """Pinned cudaMemcpyAsync H2D / D2H rates of this GPU's host link (GB/s): 1 GiB copies from
    host memory on the GPU's NUMA node, each started after a barrier, so under torchrun every
    rank copies at the same time.  Returns the median over reps (the per-GPU rate with all the
    job's links busy) and every rep."""
    from mserve_b200 import topology
    with topology.local_placement(device):
        h = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    g = torch.empty(nbytes, dtype=torch.uint8, device=device)
    out = {}
    for name in ("h2d", "d2h"):
        rates = []
        for _ in range(reps):
            torch.cuda.synchronize(device)
            barrier(world)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            if name == "h2d":
                g.copy_(h, non_blocking=True)
            else:
                h.copy_(g, non_blocking=True)
            e1.record()
            e1.synchronize()
            rates.append(nbytes / (e0.elapsed_time(e1) * 1e-3) / 1e9)
        out[name] = statistics.median(rates)
        out[name + "_reps"] = rates
    del h, g
    return out


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except ValueError:
            pass
    return {}


# DRAM and host-link bytes per decode layer of the qwen7b workload on one GPU, read from ncu
# captures of the kernels (dram__bytes_read.sum + dram__bytes_write.sum; for the gather the
# sysmem bytes it pulled over PCIe).  The files and the kernels they were captured on are named
# beside each number; the bench prints them as "traffic" with that source.
NCU_TRAFFIC = {
    "gather": {"link_bytes": (1048576 + 65536) * 32,
               "source": "profiles/gather_decode_qwen7b.txt (move_rows_kernel<16>, ncu --set full)"},
    "select": {"dram_bytes": 134341888 + 4309504 + 2133760,
               "source": "profiles/select_decode_qwen7b.txt (score_stream_kernel, 24 warps per SM, + topk_smem_kernel<1> "
                         "with the early stop, ncu --set full)"},
}


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


# ------------------------------------------------------------------------------------- workload data
# Every (layer, sequence, head) slice of K/V and every (layer, sequence) query row set comes from
# its own generator seed, so any split of the problem over ranks holds exactly the same numbers.
def _gen(device, *key):
    h = 0
    for k in key:
        h = (h * 1_000_003 + int(k) + 1) % (1 << 62)
    return torch.Generator(device=device).manual_seed(h)


def kv_slice(wl, layer, b, h, n, device, tag=0, t0=0):
    """K and V rows [n, D] (bf16) of KV head h of sequence b, tokens [t0, t0 + n) of stream `tag`
    (0: the prefilled context, 1: the append turn)."""
    g = _gen(device, wl["seed"], tag, layer, b, h)
    D = wl["head_dim"]
    k = torch.randn(n, D, generator=g, device=device)
    v = torch.randn(n, D, generator=g, device=device)
    if tag == 0:
        n_img = int(wl["seq_len"] * wl["image_frac"])
        k[max(n_img - t0, 0):] *= 0.5
        v[max(n_img - t0, 0):] *= 0.5
    else:
        img = wl.get("turn_image", 0)
        k[img:] *= 0.5
        v[img:] *= 0.5
    return k.to(torch.bfloat16), v.to(torch.bfloat16)


def q_rows(wl, layer, b, device, tag=2):
    """Query rows [Hq, D] (bf16) of sequence b at one layer."""
    g = _gen(device, wl["seed"], tag, layer, b)
    return torch.randn(wl["q_heads"], wl["head_dim"], generator=g, device=device).to(torch.bfloat16)


def layer_kv(wl, layer, bs, hs, lens, device, tag=0, n=None):
    """[len(bs), len(hs), Tmax, D] K and V of the given sequences and KV heads (rows past a
    sequence's length are zero)."""
    Tmax = max(lens) if n is None else n
    K = torch.zeros(len(bs), len(hs), Tmax, wl["head_dim"], dtype=torch.bfloat16, device=device)
    V = torch.zeros_like(K)
    for i, b in enumerate(bs):
        nb = lens[b] if n is None else n
        for j, h in enumerate(hs):
            K[i, j, :nb], V[i, j, :nb] = kv_slice(wl, layer, b, h, nb, device, tag=tag)
    return K, V


def build_engine(wl, plan, device):
    """The rank's OffloadKV with its (sequence, KV head) share of the workload, and its queries
    [L, Bl, Hql, D]."""
    from mserve_b200.engine import OffloadKV
    L, Hq, Hkv, D = wl["layers"], wl["q_heads"], wl["kv_heads"], wl["head_dim"]
    G = Hq // Hkv
    bs, hs = list(range(plan.b0, plan.b1)), list(range(plan.h0, plan.h1))
    lens = workload_lens(wl)
    turn = wl.get("turn_image", 0) + wl.get("turn_text", 0)
    eng = OffloadKV(L, len(bs), len(hs) * G, len(hs), D, wl["seq_len"] + 256 + turn, top_k=wl["top_k"],
                    recent=wl["recent"], top_k_ratio=wl.get("top_k_ratio"), device=device)
    eng.reserve([lens[b] for b in bs])
    for layer in range(L):
        K, V = layer_kv(wl, layer, bs, hs, lens, device)
        eng.append_layer(layer, K, V)
        del K, V
    eng.commit()
    q = torch.stack([torch.stack([q_rows(wl, layer, b, device)[plan.h0 * G:plan.h1 * G] for b in bs])
                     for layer in range(L)])
    torch.cuda.synchronize(device)
    return eng, q


def gathered_bytes(eng):
    """Selected K+V bytes per decode layer: per segment min(k_b, L_b - R) + min(R, L_b) rows."""
    lens = eng.len_h.astype(np.int64)
    n = np.maximum(lens - eng.recent, 0)
    k = eng.topk_h if eng.top_k_ratio is not None else np.full(eng.B, eng.top_k, dtype=np.int64)
    rows = int((np.minimum(k, n) + (lens - n)).sum()) * eng.Hkv
    return 2 * rows * eng.D * torch.empty((), dtype=eng.dtype).element_size()


def append_turn(eng, wl, plan, device):
    """Appends one turn (image then text tokens) to every sequence of every layer, timed with CUDA
    events: returns (ms, bytes written to the host store, bytes written to HBM key pages)."""
    n = wl.get("turn_image", 0) + wl.get("turn_text", 0)
    bs, hs = list(range(plan.b0, plan.b1)), list(range(plan.h0, plan.h1))
    rows = [layer_kv(wl, layer, bs, hs, None, device, tag=1, n=n) for layer in range(eng.L)]
    torch.cuda.synchronize(device)
    eng.reserve([n] * eng.B)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for layer, (k, v) in enumerate(rows):
        eng.append_layer(layer, k, v)
    e1.record()
    e1.synchronize()
    eng.commit()
    es = torch.empty((), dtype=eng.dtype).element_size()
    return e0.elapsed_time(e1), 2 * eng.L * eng.B * eng.Hkv * n * eng.D * es, eng.L * eng.B * eng.Hkv * n * eng.D * es


def workload_config(wl, name, world, plan_desc):
    """The `config` of both arms' lines (the reference arm prints the same one)."""
    return {"workload": name, "global_batch": wl["batch"], "seq_len": wl["seq_len"], "layers": wl["layers"],
            "parallelism": plan_desc,
            "l2": f"inputs larger than L2: {wl['layers']} layers of HBM keys and host KV read per step"}


def link_weighted_plan(wl, world, rank, h2d_ranks):
    """This rank's share of the workload given every rank's concurrent H2D link rate (GB/s):
    (plan, sequence-group weights or None, sequences per group, the job's GB/s bound).  For
    equal-length batches parallel.plan_for_links picks the head-group count and sizes each
    sequence group by the slowest rate among its ranks; ragged batches keep the even split (the
    bound then assumes every rank moves its share at the slowest rate)."""
    from mserve_b200 import parallel
    if "lens_uniform" not in wl:
        return parallel.plan_for_links(wl["batch"], wl["kv_heads"], world, rank, h2d_ranks)
    plan = parallel.shard_plan(wl["batch"], wl["kv_heads"], world, rank)
    return plan, None, [wl["batch"] // plan.seq_groups] * plan.seq_groups, world * min(h2d_ranks)


def plan_description(wl, world):
    from mserve_b200.parallel import shard_plan
    p = shard_plan(wl["batch"], wl["kv_heads"], world, 0)
    if world == 1:
        return (f"1 rank: all {wl['kv_heads']} KV heads x {wl['batch']} sequences, gathering over its own host link")
    if "lens_uniform" in wl:
        return (f"{world} ranks split one problem: {p.h1 - p.h0} of {wl['kv_heads']} KV heads x {p.b1 - p.b0} of "
                f"{wl['batch']} sequences per rank, each rank gathering over its own host link, no collective on "
                "the data path")
    return (f"{world} ranks split one problem over KV-head groups and sequence groups chosen from the ranks' "
            f"measured concurrent host-link rates (by default {p.head_groups} head groups of {p.h1 - p.h0} of "
            f"{wl['kv_heads']} KV heads, each sequence group taking sequences in proportion to its slowest link; "
            "evenly when the links are equally fast), each rank gathering over its own host link, no collective on "
            "the data path")


# ------------------------------------------------------------------------------------- CPU path
def cpu_decode_sample(eng_host, wl, layers, nthreads, h2d_device=None):
    """Runs the C restatement of the decode step on `layers` layers; returns seconds per layer
    and a per-phase breakdown.  eng_host: list of (host_k, host_v) numpy bf16 [B,Hkv,C,D] and
    q numpy [L,B,Hq,D]."""
    import ctypes as C
    from oracle import build_oracle
    lib = build_oracle.load()
    hk_list, hv_list, qn = eng_host
    B, Hq, Hkv, D, T = wl["batch"], wl["q_heads"], wl["kv_heads"], wl["head_dim"], wl["seq_len"]
    K, R = wl["top_k"], wl["recent"]
    S = K + R
    scores = np.empty((B * Hkv, T), dtype=np.float32)
    idx = np.empty((B * Hkv, S), dtype=np.int32)
    counts = np.empty(B * Hkv, dtype=np.int32)
    out = np.empty((B, Hq, D), dtype=np.float32)
    t = {"score": 0.0, "topk": 0.0, "gather": 0.0, "h2d": 0.0, "attention": 0.0}
    if h2d_device is not None:
        # the gather writes straight into pinned buffers, as index_select(out=pinned) does in
        # the reference's get_sparse_async (kv_cache.py:594-599), then one H2D copy each
        ks_t = torch.empty((B, Hkv, S, D), dtype=torch.int16).pin_memory()
        vs_t = torch.empty((B, Hkv, S, D), dtype=torch.int16).pin_memory()
        ks, vs = ks_t.numpy().view(np.uint16), vs_t.numpy().view(np.uint16)
        dk = torch.empty(ks_t.shape, dtype=torch.int16, device=h2d_device)
        dv = torch.empty_like(dk)
    else:
        ks = np.empty((B, Hkv, S, D), dtype=np.uint16)
        vs = np.empty_like(ks)
    for layer in layers:
        hk, hv = hk_list[layer], hv_list[layer]
        C_ = hk.shape[2]
        es = 2
        t0 = time.perf_counter()
        lib.okv_score_bf16(qn[layer].ctypes.data, hk.ctypes.data, Hkv * C_ * D, C_ * D, D, B, Hq, Hkv, T, D,
                           scores.ctypes.data, T, nthreads)
        t1 = time.perf_counter()
        lib.okv_topk(scores.ctypes.data, T, B * Hkv, Hkv, None, T, K, R, idx.ctypes.data, S, counts.ctypes.data,
                     nthreads)
        t2 = time.perf_counter()
        lib.okv_gather(hk.ctypes.data, hv.ctypes.data, Hkv * C_ * D * es, C_ * D * es, D * es, B, Hkv,
                       idx.ctypes.data, 32, Hkv * S, S, S, counts.ctypes.data, ks.ctypes.data, vs.ctypes.data,
                       D * es, nthreads)
        t3 = time.perf_counter()
        if h2d_device is not None:
            dk.copy_(ks_t, non_blocking=True)
            dv.copy_(vs_t, non_blocking=True)
            torch.cuda.synchronize(h2d_device)
        t4 = time.perf_counter()
        lib.okv_attention_bf16(qn[layer].ctypes.data, ks.ctypes.data, vs.ctypes.data, counts.ctypes.data, B, Hq,
                               Hkv, S, D, C.c_float(1.0 / math.sqrt(D)), out.ctypes.data, nthreads)
        t5 = time.perf_counter()
        t["score"] += t1 - t0
        t["topk"] += t2 - t1
        t["gather"] += t3 - t2
        t["h2d"] += t4 - t3
        t["attention"] += t5 - t4
    return sum(t.values()) / len(layers), {k: v / len(layers) * 1e3 for k, v in t.items()}


def cpu_gather_rate(hk, hv, wl, nthreads, reps=5):
    """The reference's host gather alone (torch index_select along tokens, restated in C:
    oracle_kv.c okv_gather) of one layer's selection -- K + V of top_k + recent rows per (sequence,
    KV head) -- at `nthreads` threads: median GB/s over reps."""
    from oracle import build_oracle
    lib = build_oracle.load()
    B, Hkv, D, T = wl["batch"], wl["kv_heads"], wl["head_dim"], wl["seq_len"]
    S = wl["top_k"] + wl["recent"]
    rng = np.random.default_rng(1)
    idx = np.stack([np.sort(rng.choice(T, S, replace=False)) for _ in range(B * Hkv)]).astype(np.int32)
    ks = np.empty((B, Hkv, S, D), dtype=np.uint16)
    vs = np.empty_like(ks)
    C_ = hk.shape[2]
    rates = []
    for _ in range(reps):
        t0 = time.perf_counter()
        lib.okv_gather(hk.ctypes.data, hv.ctypes.data, Hkv * C_ * D * 2, C_ * D * 2, D * 2, B, Hkv, idx.ctypes.data,
                       32, Hkv * S, S, S, None, ks.ctypes.data, vs.ctypes.data, D * 2, nthreads)
        rates.append(2 * ks.nbytes / (time.perf_counter() - t0) / 1e9)
    return statistics.median(rates)


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_model():
    try:
        for l in open("/proc/cpuinfo"):
            if l.startswith("model name"):
                return l.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def reference_host_data(wl, layers):
    """Host K/V (numpy bf16 bits [B, Hkv, T, D]) and q ([L, B, Hq, D]) of the workload's layers for
    the CPU path, generated on the host (same shapes and value distributions as the GPU arm)."""
    B, Hkv, D, T, Hq = wl["batch"], wl["kv_heads"], wl["head_dim"], wl["seq_len"], wl["q_heads"]
    g = torch.Generator().manual_seed(1234)
    n_img = int(T * wl["image_frac"])
    hk, hv = [], []
    for _ in range(layers):
        k = torch.randn(B, Hkv, T, D, generator=g)
        v = torch.randn(B, Hkv, T, D, generator=g)
        k[:, :, n_img:] *= 0.5
        v[:, :, n_img:] *= 0.5
        hk.append(k.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16))
        hv.append(v.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16))
        del k, v
    qn = torch.randn(layers, B, Hq, D, generator=g).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    return hk, hv, qn


# ------------------------------------------------------------------------------------- arms
def run_reference(args, world, rank):
    """The reference's CPU path (C restatement) on the host cores, every layer of every step;
    rank 0 only (the other ranks exit without work)."""
    if rank != 0:
        return
    wl = dict(WORKLOADS[args.workload][0])
    if args.layers:
        wl["layers"] = args.layers
    name = WORKLOADS[args.workload][1]
    base = {"metric": METRIC, "unit": "GB/s", "impl": "reference", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": workload_config(wl, name, world, plan_description(wl, world))}
    if "lens_uniform" in wl or "top_k_ratio" in wl:
        print(json.dumps({**base, "unavailable": "the C restatement covers fixed-length, fixed-k workloads only"}),
              flush=True)
        return
    L = wl["layers"]
    dev = torch.device("cuda", 0) if torch.cuda.is_available() else None
    hk, hv, qn = reference_host_data(wl, L)
    nth = cpu_threads()
    per_step, bd = [], None
    for step in range(args.warmup + args.steps):
        s, bd = cpu_decode_sample((hk, hv, qn), wl, list(range(L)), nth, h2d_device=dev)
        if step >= args.warmup:
            per_step.append(s * L)
    sec_step = statistics.mean(per_step)
    step_bytes = 2 * wl["batch"] * wl["kv_heads"] * (wl["top_k"] + wl["recent"]) * wl["head_dim"] * 2 * L
    value = step_bytes / sec_step / 1e9
    gather_rates = {"threads_1": cpu_gather_rate(hk[0], hv[0], wl, 1),
                    f"threads_{nth}": cpu_gather_rate(hk[0], hv[0], wl, nth)}
    sample = (f"every one of the {L} layers of every step (the whole workload); per layer: fp32 scores, radix "
              "top-k ∪ window, index_select gather into pinned buffers, H2D of the gathered rows, attention"
              + ("" if dev else " (no GPU: H2D omitted)"))
    line = {**base, "value": value, "ms_per_step": sec_step * 1e3,
            "cpu_baseline": {"value": value, "unit": "GB/s", "cores": nth, "kind": "port", "sample": sample,
                             "cpu": cpu_model(), "breakdown_ms_per_layer": bd,
                             "index_select_gather_gbs": gather_rates,
                             "gather_note": "the host gather alone (one layer's selected K+V rows) at 1 thread and "
                                            "at every core of the affinity mask"},
            "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def _phase_timer(dev, stream):
    """(capture, per_layer_ms) helpers: each phase of every layer captured as its own CUDA graph
    and replayed back to back, timed with CUDA events on the launching stream."""
    def capture(fn):
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            fn()                                    # warm-up: workspaces are allocated here
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side, capture_error_mode="relaxed"):
            fn()
        return g

    def per_layer_ms(g, L, reps):
        g.replay()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / (reps * L)
    return capture, per_layer_ms


def parity_check(eng, wl, plan, q, out_all, dev):
    """This rank's share of layer 0, bit for bit against the unsharded layer computed on this GPU
    from the same seeds: scores and selections of the rank's (sequence, KV head) pairs, the
    gathered K/V rows, and the attention outputs of the timed step (out_all[0])."""
    from mserve_b200 import ops
    L, B, Hq, Hkv, D = wl["layers"], wl["batch"], wl["q_heads"], wl["kv_heads"], wl["head_dim"]
    G = Hq // Hkv
    lens = [int(x) for x in eng.len_h]
    all_lens = workload_lens(wl)
    turn = wl.get("turn_image", 0) + wl.get("turn_text", 0)
    full_lens = [n + turn for n in all_lens]
    T = max(full_lens)
    # the unsharded layer 0 (context, plus the append turn if the workload has one)
    K, V = layer_kv(wl, 0, list(range(B)), list(range(Hkv)), all_lens, dev)
    if turn:
        Kt, Vt = layer_kv(wl, 0, list(range(B)), list(range(Hkv)), None, dev, tag=1, n=turn)
        K2 = torch.zeros(B, Hkv, T, D, dtype=K.dtype, device=dev)
        V2 = torch.zeros_like(K2)
        for b in range(B):
            K2[b, :, :all_lens[b]], V2[b, :, :all_lens[b]] = K[b, :, :all_lens[b]], V[b, :, :all_lens[b]]
            K2[b, :, all_lens[b]:full_lens[b]], V2[b, :, all_lens[b]:full_lens[b]] = Kt[b], Vt[b]
        K, V = K2, V2
    qf = torch.stack([q_rows(wl, 0, b, dev) for b in range(B)])
    len_t = torch.tensor(full_lens, dtype=torch.int32, device=dev)
    scores = torch.empty(B, Hkv, T, dtype=torch.float32, device=dev)
    ops.score(qf, ops.strided_rows(K, None, len_=len_t, device=dev), batch=B, kv_heads=Hkv, max_tokens=T, out=scores)
    if eng.top_k_ratio is not None:
        kvec = torch.tensor([math.ceil(eng.top_k_ratio * n) for n in full_lens], dtype=torch.int32, device=dev)
        top_k, k_bound = kvec, int(kvec.max())
    else:
        top_k, k_bound = eng.top_k, None
    # the engine's selection width, so both attentions split the rows the same way
    idx = torch.empty(B * Hkv, eng.S, dtype=torch.int32, device=dev)
    idx, cnt = ops.topk(scores.view(B * Hkv, T), top_k=top_k, recent=eng.recent, len_=len_t, len_scalar=T,
                        sel_per_batch=Hkv, k_bound=k_bound, out=idx)
    S = idx.shape[1]
    ksel = torch.empty(B, Hkv, S, D, dtype=K.dtype, device=dev)
    vsel = torch.empty_like(ksel)
    ops.gather(ops.strided_rows(K, V, len_=len_t, device=dev), idx.view(B, Hkv, S), ksel, vsel, batch=B,
               counts=cnt.view(B, Hkv))
    out_full = ops.sparse_attention(qf.unsqueeze(2), ksel, vsel, counts=cnt.view(B, Hkv))
    # the rank's own share, layer 0, through the engine (one layer, not pipelined)
    b0, b1, h0, h1 = plan.b0, plan.b1, plan.h0, plan.h1
    bufs = eng.buffers()
    ridx, rcnt = eng.select(0, q[0], bufs)
    eng.gather(0, ridx, rcnt, bufs)
    torch.cuda.synchronize(dev)
    ops.check_status(dev, "parity check")
    ok = {}
    ok["scores"] = all(torch.equal(bufs.scores[i, :, :lens[i]].view(torch.int32),
                                   scores[b, h0:h1, :lens[i]].contiguous().view(torch.int32))
                       for i, b in enumerate(range(b0, b1)))
    sel_ok, rows_ok = True, True
    for i, b in enumerate(range(b0, b1)):
        for j, h in enumerate(range(h0, h1)):
            n = int(cnt[b * Hkv + h])
            r = i * (h1 - h0) + j
            sel_ok &= int(rcnt[r]) == n and torch.equal(ridx[r, :n].long(), idx[b * Hkv + h, :n].long())
            rows_ok &= (torch.equal(bufs.k_sel[i, j, :n].view(torch.int16), ksel[b, h, :n].view(torch.int16)) and
                        torch.equal(bufs.v_sel[i, j, :n].view(torch.int16), vsel[b, h, :n].view(torch.int16)))
    ok["selections"] = bool(sel_ok)
    ok["gathered_rows"] = bool(rows_ok)
    ok["attention_outputs"] = torch.equal(out_all[0].view(torch.int16),
                                          out_full[b0:b1, h0 * G:h1 * G].contiguous().view(torch.int16))
    del K, V, ksel, vsel, scores
    ok["ok"] = all(ok.values())
    return ok


def shared_selection_timing(wl, plan, eng, q, world, dev, L_time, reps=4):
    """The reference's head-averaged selection (one index set per sequence ranked by the mean over
    all query heads, qwen-eljrte/Qwen_Transformer/attention.py:558-572) with the KV heads on the
    ranks of each sequence group: per exchange ("nccl": score rows all-gathered by NCCL; "peer":
    the score kernel stores them into the peers' buffers), the device time per layer of `reps` x
    L_time layers captured in one CUDA graph and replayed once (max over ranks), and a bit-for-
    bit check of layer 0's selection against the unsharded one computed on this GPU."""
    import torch.distributed as dist
    from mserve_b200 import ops, parallel
    B, Hq, Hkv, D = wl["batch"], wl["q_heads"], wl["kv_heads"], wl["head_dim"]
    Bl = plan.b1 - plan.b0
    T = int(eng.len_h.max())
    K = wl["top_k"] or math.ceil(wl["top_k_ratio"] * T)
    R = wl["recent"]
    groups = [dist.new_group(plan.group_ranks(s)) for s in range(plan.seq_groups)] if plan.seq_groups > 1 else None
    group = groups[plan.seq_group] if groups else None
    # the unsharded selection of layer 0 on this GPU: all heads of this rank's sequences
    lens_all = workload_lens(wl)
    turn = wl.get("turn_image", 0) + wl.get("turn_text", 0)
    bs = list(range(plan.b0, plan.b1))
    full_lens = [lens_all[b] + turn for b in range(B)]
    Kf = torch.zeros(Bl, Hkv, T, D, dtype=torch.bfloat16, device=dev)
    for i, b in enumerate(bs):
        for h in range(Hkv):
            Kf[i, h, :lens_all[b]] = kv_slice(wl, 0, b, h, lens_all[b], dev)[0]
            if turn:
                Kf[i, h, lens_all[b]:full_lens[b]] = kv_slice(wl, 0, b, h, turn, dev, tag=1)[0]
    qf = torch.stack([q_rows(wl, 0, b, dev) for b in bs])
    lt = torch.tensor([full_lens[b] for b in bs], dtype=torch.int32, device=dev)
    sf = torch.empty(Bl, Hkv, T, dtype=torch.float32, device=dev)
    ops.score(qf, ops.strided_rows(Kf, None, len_=lt, device=dev), batch=Bl, kv_heads=Hkv, max_tokens=T, out=sf)
    ref_idx, ref_cnt = ops.topk(sf, top_k=K, recent=R, len_=lt, len_scalar=T, rows_per_sel=Hkv, sel_per_batch=1,
                                scale=1.0 / Hq)
    torch.cuda.synchronize(dev)
    del Kf, sf
    res = {"shape": f"{Bl} sequences per sequence group, top-{K} + last {R} per sequence of the scores summed over "
                    f"all {Hq} query heads / {Hq} (the reference's mean), {plan.head_groups} rank(s) per group",
           "exchanged_bytes_per_rank_per_layer": Bl * (plan.h1 - plan.h0) * T * 4 * (plan.head_groups - 1)}
    stream = torch.cuda.current_stream(dev)
    for ex in ("nccl", "peer"):
        sel = parallel.SharedSelection(Bl, Hkv, Hq, T, group=group, device=dev, exchange=ex)
        out = torch.empty(Bl, K + R, dtype=torch.int32, device=dev)
        cnt = torch.empty(Bl, dtype=torch.int32, device=dev)

        def one(layer):
            keys = ops.paged_rows(eng.pool_k[layer], None, eng.page_table, len_=eng.lens)
            sel.select(q[layer], keys, top_k=K, recent=R, len_=eng.lens, len_scalar=T, out=out, counts=cnt)
        for _ in range(2):
            for layer in range(L_time):
                one(layer)
        torch.cuda.synchronize(dev)
        sel.check_status(f"shared selection ({ex})")
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, capture_error_mode="relaxed"):
            for _ in range(reps):
                for layer in range(L_time):
                    one(layer)
        torch.cuda.synchronize(dev)
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        g.replay()                   # once: the peer exchange's epochs were fixed at capture
        e1.record(stream)
        torch.cuda.synchronize(dev)
        sel.check_status(f"shared selection ({ex})")
        us = max_over_ranks(e0.elapsed_time(e1) * 1e3 / (reps * L_time), world)
        del g
        one(0)
        torch.cuda.synchronize(dev)
        sel.check_status(f"shared selection ({ex})")
        same = bool(torch.equal(cnt, ref_cnt) and all(torch.equal(out[i, :int(cnt[i])], ref_idx[i, :int(cnt[i])])
                                                      for i in range(Bl)))
        res[ex] = {"us_per_layer": us, "parity_ok_ranks": int(sum_over_ranks(float(same), world)), "ranks": world}
        barrier(world)
        sel.close()
    if groups:
        for gr in groups:
            dist.destroy_process_group(gr)
    return res


def extra_qwen32b(world, rank, dev, steps, warmup, chunks, h2d_ranks, layers=4):
    """The Qwen2.5-VL-32B decode shape (16 x 32768 tokens, 40/8 heads, top-4096 + last 256), split
    over the ranks like the main workload (link_weighted_plan), `layers` of its 64 layers: whole-job
    GB/s and step ms (max over ranks) of the captured step."""
    from mserve_b200 import ops
    wl = dict(WORKLOADS["qwen32b"][0], layers=layers)
    plan, _, counts, _ = link_weighted_plan(wl, world, rank, h2d_ranks)
    eng, q = build_engine(wl, plan, dev)
    out = torch.empty((wl["layers"],) + tuple(eng.buffers().out.shape), dtype=eng.dtype, device=dev)
    g = eng.capture_decode_step(q, out, chunks=chunks)
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize(dev)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        g.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    barrier(world)
    ops.check_status(dev, "32B-shape decode")
    t = max_over_ranks(e0.elapsed_time(e1) * 1e-3, world)
    total = sum_over_ranks(gathered_bytes(eng) * wl["layers"] * steps, world)
    del g, eng, q, out
    torch.cuda.empty_cache()
    return {"value": total / t / 1e9, "unit": "GB/s", "ms_per_step": t / steps * 1e3, "layers": wl["layers"],
            "of_layers": 64, "steps": steps,
            "shard": {"kv_heads_per_rank": plan.h1 - plan.h0, "sequences_per_rank": plan.b1 - plan.b0,
                      "head_groups": plan.head_groups, "sequences_per_group": counts},
            "workload": WORKLOADS["qwen32b"][1] + f" ({layers} of its 64 layers)"}


def extra_llava34b(world, rank, dev, steps, warmup, chunks, layers=2):
    """The LLaVA-v1.6-34B multi-turn shape (32 sequences of 4096-65536 tokens, 56/8 heads), its KV
    heads split over the ranks like the main workload, `layers` of its 60 layers: one timed append
    turn of 2880 image + 64 text tokens per sequence (16-token HBM key pages and host
    write-through), then the captured decode step selecting the top ceil(10% of L_b) per
    (sequence, KV head); whole-job GB/s and ms (max over ranks)."""
    from mserve_b200 import ops, parallel
    wl = dict(WORKLOADS["llava34b"][0], layers=layers)
    plan = parallel.shard_plan(wl["batch"], wl["kv_heads"], world, rank)
    eng, q = build_engine(wl, plan, dev)
    ms, host_bytes, _ = append_turn(eng, wl, plan, dev)
    t_turn = max_over_ranks(ms * 1e-3, world)
    host_all = sum_over_ranks(host_bytes, world)
    out = torch.empty((wl["layers"],) + tuple(eng.buffers().out.shape), dtype=eng.dtype, device=dev)
    g = eng.capture_decode_step(q, out, chunks=chunks)
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize(dev)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        g.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    barrier(world)
    ops.check_status(dev, "34B-shape decode")
    t = max_over_ranks(e0.elapsed_time(e1) * 1e-3, world)
    total = sum_over_ranks(gathered_bytes(eng) * wl["layers"] * steps, world)
    del g, eng, q, out
    torch.cuda.empty_cache()
    return {"value": total / t / 1e9, "unit": "GB/s", "ms_per_step": t / steps * 1e3, "layers": wl["layers"],
            "of_layers": 60, "steps": steps,
            "append_turn": {"ms": t_turn * 1e3, "host_write_bytes": host_all, "host_write_gbs": host_all / t_turn / 1e9},
            "shard": {"kv_heads_per_rank": plan.h1 - plan.h0, "sequences_per_rank": plan.b1 - plan.b0},
            "workload": WORKLOADS["llava34b"][1] + f" ({layers} of its 60 layers)"}


def extra_transfer_points(world, dev, peaks):
    """Points of the transfer sweep (one token-major layer [131072, 8, 128], whole-token rows,
    uniform-random selections, seed 4) on every rank at once: gather host->HBM and write-back
    HBM->host, each transfer replayed as a CUDA graph; GB/s over all ranks (time = slowest rank)
    against the ranks' concurrent memcpy peaks."""
    from mserve_b200 import ops
    from mserve_b200.benchmark_kv_transfer import graph_timed, structured_indices
    T, H, D = 131072, 8, 128
    gen = torch.Generator().manual_seed(4)
    pts = []
    for dtype in (torch.bfloat16, torch.float8_e4m3fn):
        es = torch.empty((), dtype=dtype).element_size()
        host = ops.host_empty((T, H, D), dtype)
        host.copy_(torch.randn(T, H, D, generator=gen).to(dtype))
        rows = host.view(1, 1, T, H * D)
        src = ops.strided_rows(rows, None, device=dev)
        for density in (0.05, 0.50):
            idx = structured_indices(T, int(T * density), 1, gen).to(torch.int32).to(dev)
            n = idx.numel()
            dst = torch.empty(1, 1, n, H * D, dtype=dtype, device=dev)
            barrier(world)
            ms_g = graph_timed(lambda: ops.gather(src, idx, dst, None, batch=1), 10)
            ok = torch.equal(dst[0, 0].cpu().view(torch.uint8), rows[0, 0][idx.cpu().long()].view(torch.uint8))
            ring = torch.tensor([T // 3], dtype=torch.int32, device=dev)
            wdst = ops.strided_rows(rows, None, len_scalar=T, ring_start=ring, ring_cap=T, device=dev)
            wsrc = ops.strided_rows(dst, None, device=dev)
            barrier(world)
            ms_w = graph_timed(lambda: ops.copy_rows(wsrc, wdst, batch=1, num_tokens=n, device=dev), 10)
            ops.check_status(dev, "transfer points")
            nbytes = n * H * D * es
            tg, tw = max_over_ranks(ms_g, world), max_over_ranks(ms_w, world)
            g_all, w_all = nbytes * world / (tg * 1e-3) / 1e9, nbytes * world / (tw * 1e-3) / 1e9
            pts.append({"dtype": str(dtype).replace("torch.", ""), "density": density, "rows": n,
                        "gather_gbs": g_all, "gather_frac_concurrent_h2d": g_all / peaks["h2d_sum"],
                        "writeback_gbs": w_all, "writeback_frac_concurrent_d2h": w_all / peaks["d2h_sum"],
                        "bit_exact_ranks": int(sum_over_ranks(float(ok), world))})
        del host
    return {"layer": f"[{T} tokens, {H} KV heads, {D}] token-major, uniform-random selections, every rank at once",
            "points": pts}


def run_mserve(args, world, rank, local):
    from mserve_b200 import _lib, ops, parallel, topology
    dev = torch.device("cuda", local)
    wl = dict(WORKLOADS[args.workload][0])
    if args.layers:
        wl["layers"] = args.layers
    L = wl["layers"]
    # Link rates first: with more ranks than KV heads, each sequence group takes sequences in
    # proportion to the slowest concurrent host-link rate among its ranks (equal shares would
    # all wait for the slowest link; equally fast links give the even split).
    barrier(world)
    peaks = pcie_peaks(dev, world)
    h2d_ranks = gather_objects(peaks["h2d"], world)
    plan, seq_weights, seq_split_counts, split_bound_gbs = link_weighted_plan(wl, world, rank, h2d_ranks)
    eng, q = build_engine(wl, plan, dev)
    eng.host_link_ctas = args.gather_ctas
    turn = None
    if wl.get("turn_image", 0) + wl.get("turn_text", 0):
        ms, host_bytes, page_bytes = append_turn(eng, wl, plan, dev)
        t_max = max_over_ranks(ms, world)
        host_all = sum_over_ranks(host_bytes, world)
        turn = {"ms": t_max, "host_write_bytes": host_all, "hbm_page_bytes": sum_over_ranks(page_bytes, world),
                "host_write_gbs": host_all / (t_max * 1e-3) / 1e9,
                "note": "one append turn over all layers: K rows into HBM key pages and K+V rows written "
                        "through to the pinned host store (mskv_copy_rows), CUDA events, max over ranks"}
    bufs = eng.buffers()
    numa_node = topology.numa_node(dev)
    peaks_all = {"h2d_sum": sum_over_ranks(peaks["h2d"], world), "d2h_sum": sum_over_ranks(peaks["d2h"], world),
                 "h2d_min_rank": min_over_ranks(peaks["h2d"], world),
                 "h2d_per_rank": gather_objects(round(peaks["h2d"], 2), world),
                 "note": f"per rank the median of {PEAK_REPS} pinned 1 GiB cudaMemcpyAsync copies, every copy "
                         "started after a barrier so all ranks copy at once; summed over ranks"}
    gb_layer = gathered_bytes(eng)
    key_bytes_layer = int(eng.len_h.sum()) * eng.Hkv * eng.D * 2
    stream = torch.cuda.current_stream(dev)

    # The product path: the whole decode step (all layers, chunk-pipelined over four streams)
    # captured once as a CUDA graph and replayed.
    out_all = torch.empty((L,) + tuple(bufs.out.shape), dtype=bufs.out.dtype, device=dev)
    n0 = _lib.launch_count()
    graph = eng.capture_decode_step(q, out_all, chunks=args.chunks)
    kernels_per_step = (_lib.launch_count() - n0) // 2     # warm-up run + captured run
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # clocks sampled from the warm-up through the timed region (a short timed region alone can
    # end before nvidia-smi's first sample)
    with ClockSampler(local) as clk:
        for _ in range(args.warmup):
            graph.replay()
        torch.cuda.synchronize(dev)
        ops.check_status(dev, "bench warm-up")
        barrier(world)
        torch.cuda.synchronize(dev)
        t0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        t1.record(stream)
        torch.cuda.synchronize(dev)
    barrier(world)
    launches = kernels_per_step * args.steps
    elapsed = t0.elapsed_time(t1) * 1e-3
    ops.check_status(dev, "bench")
    t_max = max_over_ranks(elapsed, world)
    total_bytes = sum_over_ranks(gb_layer * L * args.steps, world)
    value = total_bytes / t_max / 1e9
    ms_step = t_max / args.steps * 1e3

    parity = None
    if not args.no_parity:
        ok = parity_check(eng, wl, plan, q, out_all, dev)
        per_rank = gather_objects(ok, world)
        parity = {"ok": all(p["ok"] for p in per_rank), "ranks_ok": sum(p["ok"] for p in per_rank), "ranks": world,
                  "per_rank": per_rank,
                  "checked": "layer 0 on every rank: its (sequence, KV head) pairs' fp32 scores, selected indices, "
                             "gathered K/V rows and the timed step's attention outputs, bit for bit against the "
                             "unsharded layer computed on the same GPU from the same seeds"}

    # Per-kernel durations for the rooflines: each phase of every layer -- scores + top-k, the
    # gather, the attention -- captured as its own CUDA graph and replayed back to back, timed
    # with CUDA events on the launching stream (no other phase runs beside it).
    capture, per_layer_ms = _phase_timer(dev, stream)
    reps = max(3, 84 // L)
    g_sel = capture(lambda: [eng.select(layer, q[layer], bufs) for layer in range(L)])
    sel_ms = per_layer_ms(g_sel, L, reps)
    g_gat = capture(lambda: [eng.gather(layer, bufs.idx, bufs.counts, bufs) for layer in range(L)])
    gat_ms = per_layer_ms(g_gat, L, reps)
    g_att = capture(lambda: [eng.attend(q[layer], bufs.counts, bufs) for layer in range(L)])
    att_ms = per_layer_ms(g_att, L, reps)
    del g_sel, g_gat, g_att
    serial_ms_step = L * (sel_ms + gat_ms + att_ms)
    ops.check_status(dev, "bench phase timing")
    gat_ms_max = max_over_ranks(gat_ms, world)
    gat_ms_ranks = gather_objects(round(gat_ms, 5), world)

    # end to end through the public API: q from pinned host each step, outputs back to host
    e2e = None
    if not args.no_e2e:
        q_host = q.cpu().pin_memory()
        out_host = torch.empty(out_all.shape, dtype=out_all.dtype).pin_memory()

        def e2e_step():
            q.copy_(q_host, non_blocking=True)
            graph.replay()
            out_host.copy_(out_all, non_blocking=True)
            torch.cuda.current_stream(dev).synchronize()
        for _ in range(min(args.warmup, 3)):
            e2e_step()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        barrier(world)
        te = max_over_ranks(e0.elapsed_time(e1) * 1e-3, world)
        e2e = {"value": total_bytes / te / 1e9, "unit": "GB/s", "ms_per_step": te / args.steps * 1e3,
               "h2d_bytes_per_step": int(sum_over_ranks(q_host.numel() * q_host.element_size(), world)),
               "d2h_bytes_per_step": int(sum_over_ranks(out_host.numel() * out_host.element_size(), world)),
               "api": "OffloadKV.capture_decode_step graph (score, top-k, gather, attention for all layers), "
                      "q copied H2D from pinned host and outputs D2H every step on every rank"}

    # The shared (head-averaged) selection with the heads on the ranks: both exchanges.
    shared = None
    if not args.no_exchange:
        import torch.distributed as dist
        own_group = False
        if world == 1:           # a one-rank process group, so the same code runs at every N
            dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{free_port()}", rank=0, world_size=1,
                                    timeout=datetime.timedelta(seconds=60), device_id=dev)
            own_group = True
        try:
            shared = shared_selection_timing(wl, plan, eng, q, world, dev, L_time=min(L, 8))
        finally:
            if own_group:
                dist.destroy_process_group()

    # The 32B shape, the 34B multi-turn shape and transfer-sweep points on the same ranks.
    extra = None
    if not args.no_extra:
        extra = {"qwen32b_decode": extra_qwen32b(world, rank, dev, args.steps, args.warmup, args.chunks, h2d_ranks),
                 "llava34b_decode": extra_llava34b(world, rank, dev, args.steps, args.warmup, args.chunks),
                 "transfer": extra_transfer_points(world, dev, peaks_all)}

    # CPU baseline: the C restatement on this host's cores, rank 0 at N=1 only
    cpu = None
    fixed_shape = "lens_uniform" not in wl and "top_k_ratio" not in wl   # what the C port restates
    if rank == 0 and world == 1 and not args.no_cpu_baseline and fixed_shape:
        nth = cpu_threads()
        hk = [t.view(torch.int16).numpy().view(np.uint16) for t in eng.host_k]
        hv = [t.view(torch.int16).numpy().view(np.uint16) for t in eng.host_v]
        qn = q.cpu().view(torch.int16).numpy().view(np.uint16)
        sample_layers = list(range(min(4, L)))
        reps_cpu = []
        cpu_t0 = time.perf_counter()
        for r in range(12):          # one untimed pass, then timed passes until ~10 s of CPU work
            s, bd = cpu_decode_sample((hk, hv, qn), wl, sample_layers, nth, h2d_device=dev)
            if r:
                reps_cpu.append((s, bd))
            if r >= 2 and time.perf_counter() - cpu_t0 > 10.0:
                break
        s = statistics.mean(x[0] for x in reps_cpu)
        cpu = {"value": gb_layer / s / 1e9, "unit": "GB/s", "cores": nth, "kind": "port",
               "sample": f"layers 0-{len(sample_layers) - 1} of the same host store, {len(reps_cpu)} timed passes; "
                         "per layer: fp32 scores, radix top-k ∪ window, index_select gather, H2D of the gathered "
                         "rows, attention",
               "ms_per_layer": s * 1e3, "breakdown_ms": reps_cpu[-1][1], "cpu": cpu_model(),
               "index_select_gather_gbs": {"threads_1": cpu_gather_rate(hk[0], hv[0], wl, 1),
                                           f"threads_{nth}": cpu_gather_rate(hk[0], hv[0], wl, nth)}}

    # A decode loop whose step writes its own token into every layer (HBM key page + host
    # store): begin_step() grows the lengths, then the step captured with k_new/v_new and a
    # length bound is replayed.  Run last: it grows the cache.
    loop = None
    n_loop = min(args.steps, eng.C - int(eng.len_h.max()) - args.warmup - 1)
    if not args.no_decode_loop and n_loop > 0:
        B, Hkv, D = eng.B, eng.Hkv, eng.D
        k_new = torch.stack([torch.stack([q_rows(wl, layer, b, dev, tag=3)[plan.h0:plan.h1]
                                          for b in range(plan.b0, plan.b1)]) for layer in range(L)])
        v_new = torch.stack([torch.stack([q_rows(wl, layer, b, dev, tag=4)[plan.h0:plan.h1]
                                          for b in range(plan.b0, plan.b1)]) for layer in range(L)])
        t_bound = int(eng.len_h.max()) + args.warmup + n_loop + 1
        eng.begin_step()
        n0 = _lib.launch_count()
        g_loop = eng.capture_decode_step(q, out_all, chunks=args.chunks, k_new=k_new, v_new=v_new,
                                         t_bound=t_bound)
        loop_kernels = (_lib.launch_count() - n0) // 2
        for _ in range(args.warmup):
            eng.begin_step()
            g_loop.replay()
        torch.cuda.synchronize(dev)
        barrier(world)
        loop_bytes = 0
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n_loop):
            eng.begin_step()
            loop_bytes += gathered_bytes(eng) * L
            g_loop.replay()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        barrier(world)
        ops.check_status(dev, "bench decode loop")
        tl = max_over_ranks(e0.elapsed_time(e1) * 1e-3, world)
        loop = {"value": sum_over_ranks(loop_bytes, world) / tl / 1e9, "unit": "GB/s",
                "ms_per_step": tl / n_loop * 1e3, "steps": n_loop, "kernels_per_step": loop_kernels,
                "tokens_appended_per_step": wl["batch"],
                "host_write_bytes_per_step": int(sum_over_ranks(2 * L * B * Hkv * D * 2, world)),
                "note": "each step: begin_step() on the host (lengths, splits, new pages through pinned "
                        "staging), then the captured step, which writes its token into every layer's HBM "
                        "key page and host store before that layer's selection; CUDA events around the loop"}
        del g_loop

    peaks_json = measured_peaks()
    gather_gbs = gb_layer / (gat_ms * 1e-3) / 1e9
    roofline = {"bound": "host_link", "kernel": "move_rows_kernel (mskv_gather)", "achieved": gather_gbs,
                "peak": peaks["h2d"], "unit": "GB/s", "frac": gather_gbs / peaks["h2d"],
                "peak_source": f"pinned cudaMemcpyAsync H2D of this rank's link, median of {PEAK_REPS} x 1 GiB, "
                               "measured in this run with every rank copying at once",
                "algorithmic_bytes_per_launch": gb_layer,
                "traffic": NCU_TRAFFIC["gather"]["link_bytes"] if (world == 1 and args.workload == "qwen7b") else None,
                "traffic_kind": "bytes read over the host link (sysmem), one ncu capture",
                "traffic_source": NCU_TRAFFIC["gather"]["source"],
                "timing": "gather kernels of all layers replayed as one CUDA graph, CUDA events, rank 0"}
    hbm_peak = peaks_json.get("hbm_gbs", 6650.0)
    score_gbs = key_bytes_layer / (sel_ms * 1e-3) / 1e9
    roofline_select = {"bound": "hbm", "kernel": "score_stream_kernel + topk_smem_kernel", "achieved": score_gbs,
                       "peak": hbm_peak, "unit": "GB/s", "frac": score_gbs / hbm_peak,
                       "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)" if "hbm_gbs" in peaks_json
                       else "fallback 6650 GB/s", "algorithmic_bytes_per_launch": key_bytes_layer,
                       "traffic": (NCU_TRAFFIC["select"]["dram_bytes"]
                                   if (world == 1 and args.workload == "qwen7b") else None),
                       "traffic_source": NCU_TRAFFIC["select"]["source"],
                       "timing": "score + top-k kernels of all layers replayed as one CUDA graph, CUDA events, rank 0"}
    if rank == 0:
        name = WORKLOADS[args.workload][1]       # config["layers"] carries a --layers override
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": workload_config(wl, name, world, plan_description(wl, world)),
            "shard": {"kv_heads_per_rank": plan.h1 - plan.h0, "sequences_per_rank": plan.b1 - plan.b0,
                      "head_groups": plan.head_groups, "sequence_groups": plan.seq_groups,
                      "sequences_per_group": seq_split_counts,
                      "sequence_split": ("in proportion to each sequence group's slowest concurrent H2D link rate "
                                         f"{[round(x, 2) for x in seq_weights]} GB/s") if seq_weights else "even"},
            "parity": parity,
            "roofline": roofline, "roofline_select": roofline_select,
            "breakdown_ms_per_layer": {"score_topk": sel_ms, "gather": gat_ms, "gather_max_over_ranks": gat_ms_max,
                                       "gather_per_rank": gat_ms_ranks,
                                       "attention": att_ms,
                                       "note": "rank 0's share; each phase of all layers replayed alone as a CUDA "
                                               "graph after the timed region; the attention then reads its rows "
                                               "from L2"},
            "serial_ms_per_step": serial_ms_step, "chunks": args.chunks, "gather_ctas": args.gather_ctas or "default",
            "append_turn": turn,
            "pcie_peak_gbs": peaks,
            "pcie_peak_gbs_all_ranks": peaks_all,
            "gather_frac_of_concurrent_h2d_peak_whole_step": value / peaks_all["h2d_sum"],
            # equal shares finish with the slowest rank: its concurrent link rate x N bounds the job
            "gather_frac_of_slowest_rank_peak_x_n": value / (peaks_all["h2d_min_rank"] * world),
            # the job's bound for the split it ran: every group's ranks move its share at the
            # group's slowest link rate, and the slowest group sets the step
            "gather_frac_of_split_bound": value / split_bound_gbs,
            "host_placement": {"numa_node": numa_node, "local_cpus": len(eng.host_cpus),
                               "note": "host store allocated on the GPU's local CPUs (0: placement left to the system)"},
            "shared_selection": shared,
            "extra_workloads": extra,
            "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": int(launches), "decode_loop": loop,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)


def main():
    args = parse()
    world, rank, local = dist_setup(args.gpus)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_mserve(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
