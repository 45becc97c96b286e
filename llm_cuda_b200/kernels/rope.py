"""Fused RoPE-on-new-tokens + KV-page append (CUDA, ``llmc_rope_append``).

Replaces the reference's per-step ``build_rope_cache`` + ``apply_rotary``
(``src/llm_cuda/models/llama3/attention.py:110-119``, ``kernels/triton/rope.py:156-222``)
and ``PagedKVLayerCache.append`` (``models/llama3/kv_cache.py:38-63``) with one launch.
"""

from __future__ import annotations

import torch

from .. import _native as N


def rope_append(
    q: torch.Tensor | None,
    k: torch.Tensor,
    v: torch.Tensor,
    key_pages: torch.Tensor,
    value_pages: torch.Tensor,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    status: torch.Tensor,
    cos: torch.Tensor | None = None,
    sin: torch.Tensor | None = None,
    q_out: torch.Tensor | None = None,
) -> torch.Tensor | None:
    """Rotate q/k of S new tokens per sequence, write k/v into the pages, advance seq_lens.

    Shapes: ``q [B, Hq, S, d]`` (optional), ``k``/``v`` ``[B, Hkv, S, d]``, pages
    ``[num_pages, Hkv, P, d]``, ``block_table [B, max_pages]`` int32, ``seq_lens [B]``
    int32 (positions of token 0; advanced by S on the device), ``cos``/``sin``
    ``[max_pos, d]`` (``None``: plain append of already-rotated k).  Returns the
    rotated q (``q_out`` if given) or ``None``.
    """
    lib = N.load()
    B, Hkv, S, d = k.shape
    if v.shape != k.shape:
        raise ValueError("k and v shapes must match")
    if key_pages.dtype != k.dtype or value_pages.dtype != k.dtype:
        raise ValueError("page dtype must match k/v dtype")
    if not (k.is_cuda and key_pages.is_cuda):
        raise ValueError("rope_append needs CUDA tensors")
    num_pages, Hkv_p, P, d_p = key_pages.shape
    if (Hkv_p, d_p) != (Hkv, d):
        raise ValueError("k/v shapes do not match cache layout")
    if block_table.dtype != torch.int32 or seq_lens.dtype != torch.int32:
        raise ValueError("block_table and seq_lens must be int32")
    k = k.contiguous()
    v = v.contiguous()
    Hq = 0
    if q is not None:
        q = q.contiguous()
        Hq = q.shape[1]
        if q.shape[0] != B or q.shape[2] != S or q.shape[3] != d or q.dtype != k.dtype:
            raise ValueError("q must be [B, Hq, S, d] in the k dtype")
        if q_out is None:
            q_out = torch.empty_like(q)
    rope_max = 0
    if cos is not None:
        if sin is None or cos.shape != sin.shape or cos.shape[-1] != d or cos.dtype != k.dtype:
            raise ValueError("cos/sin must be [max_pos, d] in the k dtype")
        cos = cos.contiguous()
        sin = sin.contiguous()
        rope_max = cos.shape[0]
    rc = lib.llmc_rope_append(
        N.ptr(q), k.data_ptr(), v.data_ptr(), N.ptr(q_out), key_pages.data_ptr(),
        value_pages.data_ptr(), block_table.data_ptr(), seq_lens.data_ptr(), N.ptr(cos), N.ptr(sin),
        B, S, Hq, Hkv, d, P, block_table.shape[1], num_pages, rope_max, N.dtype_code(k.dtype),
        status.data_ptr(), N.stream_handle(k.device))
    N.check(rc, "llmc_rope_append")
    return q_out
