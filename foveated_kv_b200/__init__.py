"""foveated_kv_b200 -- FoveatedKV decode hot path on NVIDIA B200 (sm_100a).

Python surface mirroring the reference package (samfurr/foveated_kv):
tier config, cache/compress entry point, fused per-layer decode attention
with spike flags, and the promotion pipeline, all backed by libfkv.so.
"""

from .config import TierConfig, MLXTierConfig
from .cache import FoveatedLayer, FoveatedKVCache, MLXFoveatedLayer, MLXFoveatedKVCache, compress_layer
from ._native import FkvNativeError
from .promotion import PromotionPipeline
from .disk_archive import DiskArchive, create_disk_archive, offload_cache_to_disk

__all__ = ["TierConfig", "MLXTierConfig", "FoveatedLayer", "FoveatedKVCache",
           "MLXFoveatedLayer", "MLXFoveatedKVCache", "compress_layer", "FkvNativeError", "PromotionPipeline",
           "DiskArchive", "create_disk_archive", "offload_cache_to_disk"]
