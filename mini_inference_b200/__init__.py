"""B200-native (sm_100a) paged-KV hot path for mini-inference.

A drop-in for the reference's ``engine/kv_cache.py`` paged cache and the
attention calls that read and write it. Host code is Python over a C ABI
(``include/pkv.h``, ``libpkv.so``): a C++ block manager with the reference's
allocation and prefix-cache decisions, and hand-written CUDA kernels for the
KV append, paged decode attention, varlen paged prefill attention, the
metadata builder and block copy-on-write. Importing the package loads
``libpkv.so``; without it the import fails (there is no CPU fallback).
"""

from ._lib import PkvError
from .cache import NativeBlockManager, PackedPrefillContext, PagedDecodeContext, PagedKVCache
from .cuda_graphs import GraphedDecoder

__all__ = ["PagedKVCache", "PagedDecodeContext", "PackedPrefillContext", "NativeBlockManager", "GraphedDecoder",
           "PkvError"]
__version__ = "0.1.0"
