"""Llama 3 decode-path modules mirroring ``llm_cuda.models.llama3``."""

from .kv_cache import PagedKVCache, PagedKVLayerCache, make_block_table
from .rotary import RopeTable, build_inv_freq, build_rope_cache

__all__ = ["PagedKVCache", "PagedKVLayerCache", "RopeTable", "build_inv_freq",
           "build_rope_cache", "make_block_table"]
