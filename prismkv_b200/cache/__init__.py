"""prismkv_b200.cache -- the reference's prismkv.cache API on device-resident codes.

    from prismkv_b200.cache import PrismKVConfig, PrismKVBackend, RawKVCache
    from prismkv_b200.cache import PrismKVCache          # HuggingFace DynamicCache
    from prismkv_b200.cache import VLLMSwapCompressor    # vLLM swap boundary
"""

from .cache_config import PrismKVConfig
from .dim_aligner import DimAligner
from .backend import CacheBackend, PrismKVBackend
from .raw_cache import RawKVCache
from .kv_cache import PrismKVCache
from .cache_store import save_cache, load_cache
from .vllm_adapter import VLLMSwapCompressor

__all__ = ["PrismKVConfig", "DimAligner", "CacheBackend", "PrismKVBackend", "RawKVCache", "PrismKVCache",
           "save_cache", "load_cache", "VLLMSwapCompressor"]
