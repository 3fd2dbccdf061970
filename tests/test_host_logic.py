"""Host-side logic that needs no GPU: decode-step chunking, workload lengths, gathered bytes."""
from types import SimpleNamespace

import numpy as np
import pytest


def test_chunk_bounds_first_chunk_single_sequence():
    from mserve_b200.engine import OffloadKV
    cb = lambda B, n: OffloadKV.chunk_bounds(SimpleNamespace(B=B), n).tolist()
    assert cb(8, 4) == [0, 1, 3, 5, 8]
    assert cb(8, 1) == [0, 8]
    assert cb(3, 4) == [0, 1, 2, 3]
    assert cb(1, 4) == [0, 1]
    assert cb(32, 4) == [0, 1, 11, 21, 32]
    for B in range(1, 40):
        for n in range(1, 9):
            b = cb(B, n)
            assert b[0] == 0 and b[-1] == B and all(x < y for x, y in zip(b, b[1:]))
            assert len(b) - 1 == min(n, B)
            if min(n, B) > 1:
                assert b[1] == 1                     # the first chunk holds one sequence


def test_chunk_bounds_explicit_sizes():
    from mserve_b200.engine import OffloadKV
    eng = SimpleNamespace(B=8)
    assert OffloadKV.chunk_bounds(eng, [1, 3, 3, 1]).tolist() == [0, 1, 4, 7, 8]
    for bad in ([1, 2], [0, 8], [4, 5], []):
        with pytest.raises(ValueError):
            OffloadKV.chunk_bounds(eng, bad)


def test_workload_lengths_and_gathered_bytes():
    import bench
    wl = dict(bench.WORKLOADS["llava34b"][0])
    lens = bench.workload_lens(wl)
    assert len(lens) == 32 and all(4096 <= x <= 65536 for x in lens)
    assert lens == bench.workload_lens(wl)           # seeded
    assert bench.workload_lens(dict(bench.WORKLOADS["qwen7b"][0])) == [16384] * 8
    # per segment: min(k_b, L_b - R) top-k rows + min(R, L_b) window rows, K and V, 2 bytes
    eng = SimpleNamespace(len_h=np.array([100, 5, 0]), recent=8, top_k_ratio=None, top_k=50, B=3, Hkv=2,
                          D=4, topk_h=None, dtype=__import__("torch").bfloat16)
    rows = (50 + 8) + (0 + 5) + 0
    assert bench.gathered_bytes(eng) == 2 * rows * 2 * 4 * 2
    eng.top_k_ratio, eng.topk_h = 0.1, np.array([10, 1, 0])
    rows = (10 + 8) + (0 + 5) + 0
    assert bench.gathered_bytes(eng) == 2 * rows * 2 * 4 * 2


def test_reference_arm_json_line():
    """bench.py --impl reference on this machine's cores: one JSON line with the bench
    contract's keys, the same metric as the product arm, a cpu_baseline describing the run and
    an e2e object with no host<->device bytes."""
    import json
    import subprocess
    import sys
    from pathlib import Path

    import bench
    root = Path(bench.__file__).resolve().parent
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0",
                        "--layers", "2"], cwd=root, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [x for x in r.stdout.splitlines() if x.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC
    assert line["unit"] == "GB/s" and line["higher_is_better"] is True and line["value"] > 0
    assert line["n_gpus"] == 1 and line["steps"] == 1 and line["warmup"] == 0
    wl = dict(bench.WORKLOADS["qwen7b"][0], layers=2)
    name = bench.WORKLOADS["qwen7b"][1]
    # the same config as the product arm prints at this N
    assert line["config"] == bench.workload_config(wl, name, 1, bench.plan_description(wl, 1))
    assert line["scaling"] == "strong"
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert "every one of the 2 layers" in cb["sample"]
    assert cb["index_select_gather_gbs"]["threads_1"] > 0 and len(cb["index_select_gather_gbs"]) == 2
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_get_full_kv_host_tensors_and_oracle():
    """get_full_kv on host tensors is torch.cat, as in the reference (kv_cache.py:631-643); the
    oracle's restatement gives the same arrays; with no past the new rows come back as they are."""
    import numpy as np
    import torch
    from oracle import kv_oracle as ko
    from mserve_b200.kv_cache import CPUKVCache
    g = torch.Generator().manual_seed(2)
    past = (torch.randn(2, 3, 9, 16, generator=g), torch.randn(2, 3, 9, 16, generator=g))
    kn, vn = torch.randn(2, 3, 4, 16, generator=g), torch.randn(2, 3, 4, 16, generator=g)
    k, v = CPUKVCache.get_full_kv(past, kn, vn)
    ek, ev = ko.full_kv((past[0].numpy(), past[1].numpy()), kn.numpy(), vn.numpy())
    np.testing.assert_array_equal(k.numpy(), ek)
    np.testing.assert_array_equal(v.numpy(), ev)
    assert CPUKVCache.get_full_kv(None, kn, vn) == (kn, vn)


def test_link_weighted_plan():
    """The bench's split of the 7B decode problem by measured link rates: even on equal links and
    at N <= 4 (no sequence groups), 3 + 5 sequences when ranks 0-3 are slower at N = 8; the bound
    is N x the slowest rate for even splits and the slowest group's rate otherwise."""
    import bench
    wl = dict(bench.WORKLOADS["qwen7b"][0])
    plan, w, counts, bound = bench.link_weighted_plan(wl, 1, 0, [55.5])
    assert w is None and counts == [8] and (plan.b0, plan.b1, plan.h0, plan.h1) == (0, 8, 0, 4)
    assert bound == pytest.approx(55.5)
    plan, w, counts, bound = bench.link_weighted_plan(wl, 4, 2, [28.7, 28.5, 28.9, 28.8])
    assert w is None and counts == [8] and (plan.h0, plan.h1) == (2, 3) and bound == pytest.approx(4 * 28.5)
    rates = [23.4, 23.4, 23.5, 23.5, 35.9, 36.2, 35.9, 35.8]
    shares = {}
    for r in range(8):
        plan, w, counts, bound = bench.link_weighted_plan(wl, 8, r, rates)
        assert w == [23.4, 35.8] and counts == [3, 5]
        shares[r] = (plan.b0, plan.b1, plan.h0, plan.h1)
        assert bound == pytest.approx(8 * 4 / max(3 / 23.4, 5 / 35.8))
    assert shares[0] == (0, 3, 0, 1) and shares[7] == (3, 8, 3, 4)
    plan, w, counts, _ = bench.link_weighted_plan(wl, 8, 5, [30.0] * 8)
    assert counts == [4, 4] and (plan.b0, plan.b1) == (4, 8)
