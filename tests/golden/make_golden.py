"""Generates tests/golden/reference_vectors.npz by running MServe's own Python code on CPU.

Run where the reference is checked out:

    python tests/golden/make_golden.py --reference <MServe checkout>
    (or MSERVE_REFERENCE=<MServe checkout> python tests/golden/make_golden.py)

What is executed (unmodified reference source, CPU tensors):
  * compute_token_importance, sparse_sdpa_attention, repeat_kv
    (qwen-eljrte/Qwen_Transformer/attention.py:532-641, 1701-1710) -- extracted with ``ast``
    because importing attention.py pulls in matplotlib/seaborn/nvtx/cv2 and a transformers
    class (SlidingWindowCache) that this environment does not have;
  * CPUKVCache.append_new and CPUKVCache.get_sparse_async
    (qwen-eljrte/Qwen_Transformer/kv_cache.py:545-629, 718-765) -- the module is executed
    with its CUDA-only calls (stream/event creation, pin_memory) replaced by CPU stand-ins
    and its module-level ``device`` set to "cpu";
  * generate_scattered_indices (qwen-eljrte/benchmark_kv_transfer.py:59-85).
bfloat16 tensors are stored as uint16 bit patterns.  The fixture is committed; tests never
read the reference tree.
"""
from __future__ import annotations

import argparse
import os
import ast
import contextlib
import math
import sys
import types
import typing
from pathlib import Path
from unittest import mock

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent


def _bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()
    return t.contiguous().numpy().copy()


def load_attention_functions(ref: Path) -> dict:
    src = (ref / "qwen-eljrte/Qwen_Transformer/attention.py").read_text()
    tree = ast.parse(src)
    wanted = {"compute_token_importance", "sparse_sdpa_attention", "repeat_kv"}
    nodes = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in wanted]
    assert {n.name for n in nodes} == wanted, "reference functions not found"
    mod = ast.Module(body=nodes, type_ignores=[])
    ns = {"torch": torch, "math": math, "F": F, "np": np}
    ns.update({k: getattr(typing, k) for k in ("Optional", "Tuple", "List", "Dict", "Any", "Union")})
    exec(compile(mod, str(ref / "qwen-eljrte/Qwen_Transformer/attention.py"), "exec"), ns)
    return ns


class _FakeStream:
    def __init__(self, *a, **k):
        pass

    def wait_event(self, *a, **k):
        pass


class _FakeEvent:
    def __init__(self, *a, **k):
        pass

    def record(self, *a, **k):
        pass

    def synchronize(self):
        pass


@contextlib.contextmanager
def cpu_stand_ins():
    real_empty = torch.empty

    def empty(*a, **k):
        k.pop("pin_memory", None)
        return real_empty(*a, **k)

    with mock.patch.object(torch.cuda, "Stream", _FakeStream), \
            mock.patch.object(torch.cuda, "Event", _FakeEvent), \
            mock.patch.object(torch.cuda, "stream", lambda s: contextlib.nullcontext()), \
            mock.patch.object(torch, "empty", empty), \
            mock.patch.object(torch.Tensor, "pin_memory", lambda self, *a, **k: self), \
            mock.patch.object(torch.Tensor, "is_pinned", lambda self, *a, **k: True):
        yield


def load_kv_cache_class(ref: Path):
    path = ref / "qwen-eljrte/Qwen_Transformer/kv_cache.py"
    mod = types.ModuleType("reference_kv_cache")
    mod.__file__ = str(path)
    exec(compile(path.read_text(), str(path), "exec"), mod.__dict__)
    mod.device = "cpu"
    return mod.CPUKVCache


def load_index_generator(ref: Path):
    path = ref / "qwen-eljrte/benchmark_kv_transfer.py"
    tree = ast.parse(path.read_text())
    nodes = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "generate_scattered_indices"]
    ns = {"torch": torch, "np": np, "Tuple": typing.Tuple, "Optional": typing.Optional}
    exec(compile(ast.Module(body=nodes, type_ignores=[]), str(path), "exec"), ns)
    return ns["generate_scattered_indices"]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("MSERVE_REFERENCE"),
                    help="root of an MServe checkout (default: $MSERVE_REFERENCE)")
    ap.add_argument("--out", default=str(HERE / "reference_vectors.npz"))
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set MSERVE_REFERENCE to the root of an MServe checkout")
    ref = Path(args.reference)
    fx = load_attention_functions(ref)
    out: dict = {}

    # ---- compute_token_importance ------------------------------------------------------
    g = torch.Generator().manual_seed(11)
    cases = [
        # name, B, Hq, Hkv, Q, T, D, dtype, method, ratio, min_tokens
        ("cti_f64_score", 1, 4, 2, 1, 600, 16, torch.float64, "attention_score", 0.3, 128),
        ("cti_f64_norm", 1, 4, 2, 1, 600, 16, torch.float64, "norm", 0.3, 128),
        ("cti_f64_q3", 1, 6, 2, 3, 500, 32, torch.float64, "attention_score", 0.3, 128),
        ("cti_f64_short", 1, 4, 4, 1, 100, 16, torch.float64, "attention_score", 0.3, 128),
        ("cti_f64_b2", 2, 4, 1, 1, 300, 8, torch.float64, "attention_score", 0.25, 16),
        ("cti_f32_score", 1, 7, 1, 1, 1000, 64, torch.float32, "attention_score", 0.3, 128),
        ("cti_bf16_score", 1, 28, 4, 1, 1024, 64, torch.bfloat16, "attention_score", 0.3, 128),
    ]
    for name, B, Hq, Hkv, Q, T, D, dt, method, ratio, mn in cases:
        q = torch.randn(B, Hq, Q, D, generator=g, dtype=torch.float64).to(dt)
        k = torch.randn(B, Hkv, T, D, generator=g, dtype=torch.float64).to(dt)
        k_rep = fx["repeat_kv"](k, Hq // Hkv)
        idx = fx["compute_token_importance"](q, k_rep, method=method, top_k_ratio=ratio, min_tokens=mn)
        out[f"{name}/q"] = _bits(q)
        out[f"{name}/k"] = _bits(k)
        out[f"{name}/idx"] = np.sort(idx.numpy(), axis=-1)
        out[f"{name}/meta"] = np.array([B, Hq, Hkv, Q, T, D, {"attention_score": 0, "norm": 1}[method],
                                        mn], dtype=np.int64)
        out[f"{name}/ratio"] = np.array([ratio])
        out[f"{name}/dtype"] = np.array(str(dt))

    # ---- repeat_kv -------------------------------------------------------------------------
    x = torch.randn(2, 3, 5, 4, generator=g, dtype=torch.float64)
    out["repeat_kv/x"], out["repeat_kv/out"] = _bits(x), _bits(fx["repeat_kv"](x, 4))

    # ---- sparse_sdpa_attention -----------------------------------------------------------
    for name, B, Hq, Hkv, Q, S, D, dt in [("attn_f64", 2, 6, 2, 1, 40, 16, torch.float64),
                                          ("attn_bf16", 1, 28, 4, 1, 200, 128, torch.bfloat16),
                                          ("attn_f32_q2", 1, 4, 4, 2, 33, 64, torch.float32)]:
        q = torch.randn(B, Hq, Q, D, generator=g, dtype=torch.float64).to(dt)
        ks = torch.randn(B, Hkv, S, D, generator=g, dtype=torch.float64).to(dt)
        vs = torch.randn(B, Hkv, S, D, generator=g, dtype=torch.float64).to(dt)
        ks_rep, vs_rep = fx["repeat_kv"](ks, Hq // Hkv), fx["repeat_kv"](vs, Hq // Hkv)
        o = fx["sparse_sdpa_attention"](q, None, None, ks_rep, vs_rep, torch.arange(S))
        out[f"{name}/q"], out[f"{name}/k_sel"], out[f"{name}/v_sel"] = _bits(q), _bits(ks), _bits(vs)
        out[f"{name}/out"] = _bits(o)
        out[f"{name}/dtype"] = np.array(str(dt))

    # ---- CPUKVCache.append_new (cat + keep last max_len) and get_sparse_async -------------
    CPUKVCache = load_kv_cache_class(ref)
    with cpu_stand_ins():
        cache = CPUKVCache(num_layers=2, max_len=48, queue_maxsize=4)
        steps = [20, 1, 17, 30, 1, 60, 5]
        for i, n in enumerate(steps):
            k_new = torch.randn(1, 3, n, 8, generator=g, dtype=torch.float64).to(torch.bfloat16)
            v_new = torch.randn(1, 3, n, 8, generator=g, dtype=torch.float64).to(torch.bfloat16)
            cache.append_new(1, k_new, v_new)
            kc, vc, seq_len, ver = cache.get_snapshot(1)
            out[f"append/step{i}/k_new"], out[f"append/step{i}/v_new"] = _bits(k_new), _bits(v_new)
            out[f"append/step{i}/k"], out[f"append/step{i}/v"] = _bits(kc), _bits(vc)
            out[f"append/step{i}/meta"] = np.array([seq_len, ver], dtype=np.int64)
        out["append/max_len"] = np.array(48)
        cache._stop.set()
        kc, vc, seq_len, _ = cache.get_snapshot(1)
        idx = torch.tensor([5, 0, 47, 13, 13, 30, 2], dtype=torch.long)
        ks, vs, _ = cache.get_sparse_async(1, torch.device("cpu"), idx)
        out["sparse/idx"] = idx.numpy()
        out["sparse/k"], out["sparse/v"] = _bits(kc), _bits(vc)
        out["sparse/k_sel"], out["sparse/v_sel"] = _bits(ks), _bits(vs)

    # ---- benchmark index generator ---------------------------------------------------------
    gen = load_index_generator(ref)
    for seq_len, sel, seed in [(8192, 2048, 42), (4096, 100, 7)]:
        out[f"scatter/{seq_len}_{sel}_{seed}"] = gen(seq_len, sel, seed).numpy()

    np.savez_compressed(args.out, **out)
    total = sum(v.nbytes for v in out.values())
    print(f"wrote {args.out}: {len(out)} arrays, {total / 1e6:.2f} MB uncompressed")


if __name__ == "__main__":
    sys.exit(main())
