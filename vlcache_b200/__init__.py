"""vlcache_b200 — B200-native (sm_100a) warm-prefill attention path for Qwen2.5-VL.

Drop-in for the attention hot path of VLCache / nano-vllm:
  * ``vlcache_b200.layers.attention``        — ``Attention`` / ``store_kvcache``
  * ``vlcache_b200.utils.context``           — ``set_context`` / ``get_context``
  * ``vlcache_b200.layers.rotary_embedding`` — ``RotaryEmbedding`` / ``get_rope`` (RoPE of new
                                               rows, optionally fused with the KV scatter) and
                                               the M-RoPE position shift of reused image K
  * ``vlcache_b200.engine.kv_cache``         — KV-cache allocation, image-KV reuse copy,
                                               warm-prefill metadata
All compute runs in the hand-written CUDA kernels of ``libvlcache_b200.so`` (C ABI in
``include/vlcache_b200.h``); there is no CPU fallback.
"""
__version__ = "0.1.0"
