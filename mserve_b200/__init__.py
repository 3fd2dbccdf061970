"""mserve_b200: B200-native (sm_100a) KV-cache selection-and-offload path of MServe.

Public surface (mirrors the reference's plugin interface):
  mserve_b200.cuda_uva.uva_gather                    -- the ``cuda_uva`` extension
  mserve_b200.selection.compute_token_importance     -- Qwen_Transformer/attention.py
  mserve_b200.selection.sparse_sdpa_attention
  mserve_b200.selection.repeat_kv
  mserve_b200.kv_cache.CPUKVCache                    -- Qwen_Transformer/kv_cache.py
and the B200 decode engine mserve_b200.engine.OffloadKV.  All compute goes through
libmserve_kv.so (include/mserve_kv.h); importing a submodule that needs it raises
ImportError when it is not built.
"""

__all__ = ["cuda_uva", "selection", "kv_cache", "engine", "ops"]
__version__ = "0.1.0"
