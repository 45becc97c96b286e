"""Paged GQA flash-decode on B200 — drop-in for ``kernels/triton/decode_attention.py``.

Keeps the reference's entry points (``src/llm_cuda/kernels/triton/decode_attention.py``
of llm-cuda):

* ``can_use_triton_decode_attention(q, k, v, attention_mask=None)`` (:162-201) —
  same predicate, except that CUDA inputs with the native library missing raise
  instead of silently selecting a slower path;
* ``triton_decode_attention(q, k, v)`` (:204-287) — dense ``[B, Hkv, L, d]`` K/V,
  served by the paged CUDA kernel with one page per sequence;

and adds the paged entry ``paged_decode_attention(q, layer_cache)`` that reads
K/V pages in place through the block table, so ``get_kv()``'s full-cache gather
(``models/llama3/kv_cache.py:65-83``) disappears from the decode step.

Numerics follow the reference kernel: fp32 accumulation, online softmax,
``out = acc / max(l, 1e-9)`` (:154), query head ``h`` reads KV head
``h // (Hq // Hkv)`` (:90-93).  Long contexts are split into partitions whose
normalised partials are merged by a log-sum-exp kernel.
"""

from __future__ import annotations

import math

import numpy as np
import torch

from .. import _native as N

# Reference limits (decode_attention.py:28-34).
_ATTN_EPSILON: float = 1e-9
_MAX_BLOCK_D: int = 256

# partition_tokens value of the balanced split (LLMC_PARTITION_BALANCED): every SM
# takes an equal share of all rows' 64-token chunks, computed on the device.
BALANCED = 0

_PARTITION_CANDIDATES = (256, 512, 1024, 2048, 4096, 8192)
# Fixed cost of a work item in token-equivalents (pipeline fill + epilogue).
_ITEM_OVERHEAD_TOKENS = 96

_sm_count: dict[int, int] = {}


def _num_sms(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _sm_count:
        _sm_count[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _sm_count[idx]


def part_len(L: int, T: int) -> int:
    """Tokens per partition when a context of ``L`` is split at ``partition_tokens = T``:
    ``n = ceil(L / T)`` equal parts rounded up to 64 (mirrors ``part_len`` in the kernels)."""
    n = -(-L // T)
    return ((-(-L // n) + 63) // 64) * 64 if n > 0 else T


_choice_cache: dict = {}


def choose_partition_tokens(lengths, num_kv_heads: int, heads_per_kv: int, num_sms: int,
                            max_tokens: int | None = None) -> int:
    """Split-K partition length for the persistent kernel.

    Simulates the kernel's static round-robin of work items (sequence-major, then
    partition, KV head, head group) over ``num_sms`` CTAs and returns the candidate
    with the smallest busiest-CTA load; each item costs its tokens plus a fixed
    overhead, and every partition beyond the first adds a merge share.  Results are
    memoised per length vector (all layers of a step ask with the same lengths).
    """
    key = (tuple(lengths), num_kv_heads, heads_per_kv, num_sms, max_tokens)
    hit = _choice_cache.get(key)
    if hit is not None:
        return hit
    lens = np.asarray(lengths, dtype=np.int64)
    lens = lens[lens > 0]
    if lens.size == 0:
        return _PARTITION_CANDIDATES[-1]
    hg = (heads_per_kv + 7) // 8
    per_part = num_kv_heads * hg
    cap = int(max_tokens) if max_tokens else int(lens.max())
    best, best_cost = None, None
    for T in _PARTITION_CANDIDATES:
        if (cap + T - 1) // T > 4096:
            continue
        nparts = (lens + T - 1) // T
        plen = ((-(-lens // nparts)) + 63) // 64 * 64          # part_len, vectorised
        seq_of_part = np.repeat(np.arange(lens.size), nparts)
        first = np.concatenate([[0], np.cumsum(nparts)[:-1]])
        idx_in_seq = np.arange(seq_of_part.size) - first[seq_of_part]
        tok = np.minimum(plen[seq_of_part], lens[seq_of_part] - idx_in_seq * plen[seq_of_part])
        sizes = np.repeat(tok, per_part) + _ITEM_OVERHEAD_TOKENS
        load = np.bincount(np.arange(sizes.size) % num_sms, weights=sizes, minlength=num_sms)
        cost = load.max() + (8 if nparts.max() > 1 else 0)
        if best_cost is None or cost < best_cost * 0.995:
            best, best_cost = T, cost
    if len(_choice_cache) > 4096:
        _choice_cache.clear()
    _choice_cache[key] = best
    return best


class DecodeWorkspace:
    """Split-K partials (``part_o`` fp32 ``[B, Hq, max_parts, d]``, ``part_lse``).

    Allocated once and reused (nothing is allocated inside a decode step, so the
    step can be captured in a CUDA graph); grows only when a larger shape is asked.
    """

    def __init__(self, device: torch.device):
        self.device = device
        self.part_o = torch.empty(0, dtype=torch.float32, device=device)
        self.part_lse = torch.empty(0, dtype=torch.float32, device=device)
        self._counter_words = None
        self._balanced_sizes: dict = {}

    def lens_next(self, B: int) -> torch.Tensor:
        """int32 [B] scratch for the fused step's advanced lengths."""
        if getattr(self, "_lens_next", None) is None or self._lens_next.numel() < B:
            self._lens_next = torch.empty(B, dtype=torch.int32, device=self.device)
        return self._lens_next

    def get_balanced(self, B: int, Hq: int, Hkv: int, d: int):
        """Partials of the balanced split (``partition_tokens = 0``); sizes from
        ``llmc_balanced_partials_bytes`` on this device.

        ``part_lse`` starts with the kernel's per-row counters, which must be zero
        before a call; the kernel returns them to zero.  They are zeroed here when the
        buffer is new or the row count (hence the counter area) changes.
        """
        key = (B, Hq, Hkv, d)
        sizes = self._balanced_sizes.get(key)
        if sizes is None:   # one ctypes query per shape, not per call
            lse_b = N.ctypes.c_size_t(0)
            with torch.cuda.device(self.device):
                o_b = N.load().llmc_balanced_partials_bytes(B, Hq, Hkv, d, N.ctypes.byref(lse_b))
            sizes = self._balanced_sizes[key] = (o_b // 4, lse_b.value // 4)
        no, nl = sizes
        if self.part_o.numel() < no:
            self.part_o = torch.empty(no, dtype=torch.float32, device=self.device)
        if self.part_lse.numel() < nl:
            self.part_lse = torch.zeros(nl, dtype=torch.float32, device=self.device)
            self._counter_words = None
        rows = B * Hkv * ((Hq // Hkv + 7) // 8)
        words = ((rows + 1) + 31) // 32 * 32
        if self._counter_words != words:
            self.part_lse[:words].zero_()
            self._counter_words = words
        return self.part_o, self.part_lse

    def invalidate_counters(self) -> None:
        """Re-zero the balanced split's counters on next use (after a kernel gave up
        mid-step, e.g. on a wait timeout, they may be left counting)."""
        self._counter_words = None

    def get(self, B: int, Hq: int, d: int, max_parts: int):
        if max_parts <= 1:
            return None, None
        self._counter_words = None   # uniform partials overwrite the balanced counters
        no = B * Hq * max_parts * d
        nl = B * Hq * max_parts
        if self.part_o.numel() < no:
            self.part_o = torch.empty(no, dtype=torch.float32, device=self.device)
        if self.part_lse.numel() < nl:
            self.part_lse = torch.empty(nl, dtype=torch.float32, device=self.device)
        return self.part_o, self.part_lse


_workspaces: dict = {}
_status_words: dict = {}


def _default_workspace(device: torch.device) -> DecodeWorkspace:
    key = (device.type, device.index)
    if key not in _workspaces:
        _workspaces[key] = DecodeWorkspace(device)
    return _workspaces[key]


def default_status(device: torch.device) -> torch.Tensor:
    """Per-device status word used when the caller passes none."""
    key = (device.type, device.index)
    if key not in _status_words:
        _status_words[key] = torch.zeros(1, dtype=torch.int32, device=device)
    return _status_words[key]


def paged_decode(
    q: torch.Tensor,
    key_pages: torch.Tensor,
    value_pages: torch.Tensor,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    *,
    host_lens=None,
    partition_tokens: int | None = None,
    scale: float | None = None,
    out: torch.Tensor | None = None,
    workspace: DecodeWorkspace | None = None,
    status: torch.Tensor | None = None,
    force_generic: bool = False,
    events=None,
) -> torch.Tensor:
    """Decode attention of ``q [B, Hq, d]`` (or ``[B, Hq, 1, d]``) over paged K/V.

    ``host_lens`` (host copy of ``seq_lens``) only steers the partition choice; the
    kernels read the lengths on the device.  ``events``: optional pair of CUDA events
    recorded just before and just after the decode kernel (not the merge), for
    timing it on its launching stream.  Returns ``out`` shaped like ``q``.
    """
    lib = N.load()
    if not q.is_cuda:
        raise ValueError("paged_decode needs CUDA tensors")
    q_shape = q.shape
    q3 = q.reshape(q.shape[0], q.shape[1], q.shape[-1])
    if q.dim() == 4 and q.shape[2] != 1:
        raise ValueError("decode attention takes exactly one query token")
    q3 = q3.contiguous()
    B, Hq, d = q3.shape
    num_pages, Hkv, P, d_p = key_pages.shape
    if d_p != d or value_pages.shape != key_pages.shape:
        raise ValueError("q/k/v head_dim or page shapes do not match")
    if key_pages.dtype != q.dtype or value_pages.dtype != q.dtype:
        raise ValueError("q and pages must share a dtype")
    if Hq % Hkv:
        raise ValueError("n_heads must be a multiple of n_kv_heads")
    max_pages = block_table.shape[1]
    dt = N.dtype_code(q.dtype)
    if partition_tokens is None:
        if force_generic or not lib.llmc_decode_balanced_supported(
                q3.data_ptr(), key_pages.data_ptr(), value_pages.data_ptr(), dt, d, P,
                max_pages, B):
            lens = host_lens if host_lens is not None else [max_pages * P] * B
            partition_tokens = choose_partition_tokens(
                lens, Hkv, Hq // Hkv, _num_sms(q.device), max_tokens=max_pages * P)
        else:
            partition_tokens = BALANCED
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    if out is None:
        out = torch.empty_like(q3)
    ws = workspace if workspace is not None else _default_workspace(q.device)
    if partition_tokens == BALANCED:
        max_parts = 0
        part_o, part_lse = ws.get_balanced(B, Hq, Hkv, d)
    else:
        max_parts = -(-(max_pages * P) // partition_tokens)   # llmc_num_partitions
        part_o, part_lse = ws.get(B, Hq, d, max_parts)
    st = status if status is not None else default_status(q.device)
    stream = N.stream_handle(q.device)
    if events is not None:
        events[0].record()
    rc = lib.llmc_paged_decode(
        q3.data_ptr(), key_pages.data_ptr(), value_pages.data_ptr(), block_table.data_ptr(),
        seq_lens.data_ptr(), out.data_ptr(), N.ptr(part_o), N.ptr(part_lse), st.data_ptr(),
        B, Hq, Hkv, d, P, max_pages, num_pages, partition_tokens, float(scale), dt,
        N.LLMC_DECODE_FORCE_GENERIC if force_generic else 0, stream)
    N.check(rc, "llmc_paged_decode")
    if events is not None:
        events[1].record()
    rc = lib.llmc_lse_merge(N.ptr(part_o), N.ptr(part_lse), seq_lens.data_ptr(), out.data_ptr(),
                            B, Hq, d, max_parts, partition_tokens, dt, stream)
    N.check(rc, "llmc_lse_merge")
    return out.view(q_shape)


def rope_append_decode(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    key_pages: torch.Tensor,
    value_pages: torch.Tensor,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    *,
    host_lens=None,
    partition_tokens: int | None = None,
    scale: float | None = None,
    out: torch.Tensor | None = None,
    q_out: torch.Tensor | None = None,
    workspace: DecodeWorkspace | None = None,
    status: torch.Tensor | None = None,
    events=None,
    early_tables: bool = False,
) -> torch.Tensor:
    """One fused decode-attention step (``llmc_rope_append_decode``).

    ``q [B, Hq, 1, d]`` raw query, ``k``/``v`` ``[B, Hkv, 1, d]`` of the new token at
    position ``seq_lens[b]``: RoPE, the page append and the attention over
    ``seq_lens[b] + 1`` tokens run in one decode launch plus the merge launch, which
    also advances ``seq_lens``.  ``host_lens`` are the lengths BEFORE the step.
    Returns ``out`` shaped like ``q``; the rotated query goes to ``q_out``.
    ``events``: optional CUDA-event pair recorded around the step's launches.
    ``early_tables``: promise that no kernel still running when this one starts writes
    ``seq_lens``, ``block_table`` or the pages (``LLMC_DECODE_EARLY_TABLES``): the K/V
    stream then starts before the wait for the previous kernel.
    """
    lib = N.load()
    if not q.is_cuda:
        raise ValueError("rope_append_decode needs CUDA tensors")
    q_shape = q.shape
    B, Hq, d = q.shape[0], q.shape[1], q.shape[-1]
    if q.dim() == 4 and q.shape[2] != 1:
        raise ValueError("one new token per sequence")
    num_pages, Hkv, P, d_p = key_pages.shape
    if d_p != d or k.shape[0] != B or k.shape[1] != Hkv or v.shape != k.shape:
        raise ValueError("q/k/v shapes do not match the cache layout")
    if key_pages.dtype != q.dtype or k.dtype != q.dtype or cos.dtype != q.dtype:
        raise ValueError("q, k, v, pages and the RoPE table must share a dtype")
    max_pages = block_table.shape[1]
    if partition_tokens is None:
        partition_tokens = BALANCED
    # q/k/v may be views into one fused QKV projection output ([B, 1, (Hq+2Hkv)*d]
    # split into heads): read in place when only the sequence stride is not dense.
    def seq_stride(t, H):
        if t.dim() == 4 and t.shape[2] != 1:
            return None
        if t.stride(-1) != 1 or (H > 1 and t.stride(1) != d):
            return None
        return t.stride(0)
    qs, ks, vs = seq_stride(q, Hq), seq_stride(k, Hkv), seq_stride(v, Hkv)
    strided = (qs is not None and ks is not None and ks == vs and partition_tokens == BALANCED
               and ((qs, ks) != (Hq * d, Hkv * d) or early_tables)
               and lib.llmc_decode_balanced_supported(q.data_ptr(), key_pages.data_ptr(),
                                                      value_pages.data_ptr(),
                                                      N.dtype_code(q.dtype), d, P, max_pages, B))
    if not strided:
        q = q.contiguous()
        k = k.contiguous()
        v = v.contiguous()
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    out = torch.empty(B, Hq, d, dtype=q.dtype, device=q.device) if out is None else out
    q_out = torch.empty(B, Hq, d, dtype=q.dtype, device=q.device) if q_out is None else q_out
    ws = workspace if workspace is not None else _default_workspace(q.device)
    if partition_tokens == BALANCED:
        part_o, part_lse = ws.get_balanced(B, Hq, Hkv, d)
    else:
        part_o, part_lse = ws.get(B, Hq, d, -(-(max_pages * P) // partition_tokens))
    st = status if status is not None else default_status(q.device)
    if events is not None:
        events[0].record()
    args = (q.data_ptr(), k.data_ptr(), v.data_ptr(), q_out.data_ptr(), key_pages.data_ptr(),
            value_pages.data_ptr(), block_table.data_ptr(), seq_lens.data_ptr(), cos.data_ptr(),
            sin.data_ptr(), cos.shape[0], out.data_ptr(), N.ptr(part_o), N.ptr(part_lse),
            ws.lens_next(B).data_ptr(), st.data_ptr(), B, Hq, Hkv, d, P, max_pages, num_pages,
            partition_tokens, float(scale), N.dtype_code(q.dtype))
    if strided:
        flags = N.LLMC_DECODE_EARLY_TABLES if early_tables else 0
        rc = lib.llmc_rope_append_decode_strided(*args, qs, ks, flags, N.stream_handle(q.device))
    else:
        rc = lib.llmc_rope_append_decode(*args, N.stream_handle(q.device))
    if events is not None:   # brackets the decode and merge launches of the step
        events[1].record()
    N.check(rc, "llmc_rope_append_decode")
    return out.view(q_shape)


def paged_decode_attention(q: torch.Tensor, layer_cache, out: torch.Tensor | None = None,
                           partition_tokens: int | None = None) -> torch.Tensor:
    """Decode attention of ``q [B, Hq, 1, d]`` against a ``PagedKVLayerCache``."""
    return paged_decode(
        q, layer_cache.key_pages, layer_cache.value_pages, layer_cache.block_table,
        layer_cache.seq_lens, host_lens=layer_cache.host_lengths, out=out,
        partition_tokens=partition_tokens, workspace=layer_cache.workspace,
        status=layer_cache.status)


def can_use_triton_decode_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    attention_mask: torch.Tensor | None = None,
) -> bool:
    """The reference predicate (decode_attention.py:162-201) for the CUDA kernel."""
    if attention_mask is not None:
        return False
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        return False
    N.load()  # CUDA inputs but no library: fail loudly rather than fall back
    if q.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        return False
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        return False
    if q.shape[-2] != 1:
        return False
    if q.shape[0] != k.shape[0] or q.shape[0] != v.shape[0]:
        return False
    if q.shape[-1] != k.shape[-1] or q.shape[-1] != v.shape[-1]:
        return False
    if q.shape[-1] > _MAX_BLOCK_D:
        return False
    if k.shape != v.shape:
        return False
    if k.shape[-2] == 0:
        return False
    n_heads, n_kv_heads = q.shape[1], k.shape[1]
    if n_kv_heads == 0 or n_heads % n_kv_heads != 0:
        return False
    if k.dtype != q.dtype or v.dtype != q.dtype:
        return False
    return True


def triton_decode_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Flash-decode of ``q [B, Hq, 1, d]`` over dense ``k``/``v`` ``[B, Hkv, L, d]``.

    The dense cache is the paged layout with one page of ``L`` tokens per sequence
    (``[num_pages=B, Hkv, P=L, d]``), so the same CUDA kernels serve it.
    """
    B, Hkv, L, d = k.shape
    k = k.contiguous()
    v = v.contiguous()
    bt = torch.arange(B, dtype=torch.int32, device=q.device).view(B, 1)
    lens = torch.full((B,), L, dtype=torch.int32, device=q.device)
    return paged_decode(q, k, v, bt, lens, host_lens=[L] * B)
