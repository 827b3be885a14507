"""B200-native (sm_100a) sparse decode-attention path of the HeadInfer/Twilight
CPU-GPU KV-offloading prototype.

Import by path (the directory name is not a Python identifier)::

    import importlib
    tw = importlib.import_module("twilight-cpu-gpu-offloading_b200")
    cache = tw.TwilightMatchedBudgetOffloadedCache(...)

Public API mirrors the reference's offload caches (hi/quest_offload_cache.py,
hi/twilight_offload_cache.py) and its varlen attention call (hi/mp.py:21-52).
All compute runs in libtwilight_b200.so (C ABI: include/twilight_b200.h).
"""

from . import _lib, ops
from .attention import flash_attention_varlen_forward, sparse_gqa_decode_attention
from .cache import QuestTopKOffloadedCache, TwilightMatchedBudgetOffloadedCache
from .slab import MappedHostSlab, SequentialCacheState, SlabGeometry

__all__ = [
    "QuestTopKOffloadedCache",
    "TwilightMatchedBudgetOffloadedCache",
    "SlabGeometry",
    "SequentialCacheState",
    "MappedHostSlab",
    "flash_attention_varlen_forward",
    "sparse_gqa_decode_attention",
    "ops",
    "load_library",
]


def load_library():
    """Load libtwilight_b200.so (raises when it is missing; there is no fallback)."""
    return _lib.load()
