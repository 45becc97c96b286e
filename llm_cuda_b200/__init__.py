"""llm_cuda_b200 — B200-native (sm_100a) decode-attention hot path of llm-cuda.

Entry points mirror the reference's modules:

* ``llm_cuda_b200.kernels.decode_attention`` — ``can_use_triton_decode_attention``,
  ``triton_decode_attention`` and the paged ``paged_decode_attention``;
* ``llm_cuda_b200.kernels.rope`` — fused RoPE + KV-page append;
* ``llm_cuda_b200.models.llama3`` — ``PagedKVLayerCache`` / ``PagedKVCache`` with
  block tables, RoPE tables.

All compute runs in the CUDA library ``llm_cuda_b200/_lib/libllmcuda_b200.so``
(C ABI in ``include/llm_cuda_b200.h``); there is no CPU fallback.
"""

from .models.llama3.kv_cache import PagedKVCache, PagedKVLayerCache

__all__ = ["PagedKVCache", "PagedKVLayerCache"]
__version__ = "0.1.0"
