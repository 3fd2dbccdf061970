"""The oracle: a CPU restatement of MServe's KV-cache selection-and-offload path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline leg / reference arm may import, call or link anything under ``oracle/``, and
only as the checker or as the timed CPU baseline -- never as part of the product path
(``mserve_b200`` does not import it and has no CPU fallback).

Contents
  kv_oracle.py    numpy restatement, one function per reference step, each citing the
                  reference file:line it follows (qwen-eljrte/...).
  oracle_kv.c     the same gather / scoring / top-k / attention in plain C + OpenMP, used as
                  the timed CPU baseline (built into liboracle_kv.so by build_oracle.py).
  build_oracle.py gcc recipe for liboracle_kv.so.

Pinning: kv_oracle is checked against golden vectors produced by running the reference's
own Python functions (tests/golden/make_golden.py: compute_token_importance,
sparse_sdpa_attention and repeat_kv from qwen-eljrte/Qwen_Transformer/attention.py, and
CPUKVCache.append_new / get_sparse_async from qwen-eljrte/Qwen_Transformer/kv_cache.py,
executed on CPU tensors).  The reference ships no tests or fixtures of its own.
"""
