"""Kitty 2-bit KV cache - B200 (sm_100a) implementation.

Drop-in replacement for the ``kitty`` package of bitxwolf/kitty-kv: the same
public classes (``kitty/__init__.py:20-27`` there) backed by hand-written CUDA
kernels for page quantise/pack and fused paged GQA decode attention.
"""

from .config import KittyConfig
from .sensitivity import KittySensitivityProfiler
from .layout import PageCentricKVLayoutManager
from .pipeline import KittyInferencePipeline
from .attention import KittyPagedAttention, KittyAttentionFactory
from .batched import BatchedKVCache

__version__ = "0.1.0+b200"
__description__ = ("2-bit KV Cache Quantization with per-channel boosted precision and Dense-Sparse "
                   "memory decomposition; B200 CUDA kernels.")

__all__ = [
    "KittyConfig",
    "KittySensitivityProfiler",
    "PageCentricKVLayoutManager",
    "KittyInferencePipeline",
    "KittyPagedAttention",
    "KittyAttentionFactory",
    "BatchedKVCache",
]
