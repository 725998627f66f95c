"""halo_b200 -- HALO's chunked-attention hot path, B200-native (sm_100a).

Public API mirrors lzbaclz/HALO's ``halo`` package for this path:

>>> from halo_b200 import HALOConfig, wrap_with_halo
>>> model = wrap_with_halo(hf_causal_lm, HALOConfig(chunked=True, hot_ratio=0.25))

Attention runs in hand-written CUDA kernels (``libhalo_sm100.so``, C ABI in
``include/halo_b200.h``); there is no CPU fallback.
"""
from halo_b200.policy import HALOConfig, parse_overrides, wrap_with_halo
from halo_b200.scorer import HALOScorer
from halo_b200.demoter import HALODemoter
from halo_b200.refetcher import HALORefetcher
from halo_b200.kv_cache import HALOCache
from halo_b200.kv_cache_chunked import HALOCacheChunked
from halo_b200.memory_tier import MemoryTier, TieredStorage
from halo_b200.preforward_peel import install_preforward_peel

__all__ = [
    "HALOConfig",
    "parse_overrides",
    "wrap_with_halo",
    "HALOScorer",
    "HALODemoter",
    "HALORefetcher",
    "HALOCache",
    "HALOCacheChunked",
    "MemoryTier",
    "TieredStorage",
    "install_preforward_peel",
]

__version__ = "0.1.0"
