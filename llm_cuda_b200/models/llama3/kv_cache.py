"""Paged KV cache with block tables — drop-in for ``models/llama3/kv_cache.py``.

Keeps the reference's classes, constructor arguments, methods and attributes
(``src/llm_cuda/models/llama3/kv_cache.py:6-125`` of llm-cuda):
``PagedKVLayerCache(num_kv_heads, head_dim, max_seq_len, page_size, device, dtype)``
with ``append(k, v)``, ``get_kv()``, ``clear()``, ``length``, ``key_pages``,
``value_pages``, ``max_pages``; ``PagedKVCache.create(...)``, ``get_layer(i)``,
``clear()``.  Page storage keeps the reference layout
``[num_pages, num_kv_heads, page_size, head_dim]`` (kv_cache.py:28-36).

What is new (the reference is batch-1 with physical page == logical page,
kv_cache.py:43-44,55-57):

* a batch of ``batch_size`` sequences, each with its own length;
* a block table ``[batch_size, max_pages]`` (int32, on the device) mapping logical
  to physical pages of a shared pool, in any order;
* lengths live on the device (``seq_lens``) and are advanced by the append kernel
  itself, so a decode step needs no host bookkeeping and can be graph-captured;
  ``host_lengths`` mirrors them for validation and launch heuristics;
* ``append`` is one CUDA launch for all tokens and heads (the reference loops over
  tokens in Python), and ``append_rotary`` fuses RoPE into it.

``get_kv()`` still returns the gathered ``[B, Hkv, len, d]`` tensors for
compatibility; the decode path never calls it.
"""

from __future__ import annotations

import math

import torch

from ... import _native as N
from ...kernels.decode_attention import (
    DecodeWorkspace,
    paged_decode_attention,
    rope_append_decode,
)
from ...kernels.rope import rope_append
from .rotary import RopeTable


def make_block_table(batch_size: int, pages_per_seq, num_pages: int, max_pages: int,
                     generator: torch.Generator | None = None, device=None) -> torch.Tensor:
    """Block table whose sequences take pages from a shared pool in random order.

    ``pages_per_seq``: int or per-sequence list.  Unused entries are -1.
    """
    if isinstance(pages_per_seq, int):
        pages_per_seq = [pages_per_seq] * batch_size
    need = sum(pages_per_seq)
    if need > num_pages:
        raise ValueError(f"pool of {num_pages} pages cannot hold {need}")
    perm = torch.randperm(num_pages, generator=generator)[:need].to(torch.int32)
    bt = torch.full((batch_size, max_pages), -1, dtype=torch.int32)
    off = 0
    for b, n in enumerate(pages_per_seq):
        if n > max_pages:
            raise ValueError("sequence needs more pages than max_pages")
        bt[b, :n] = perm[off:off + n]
        off += n
    return bt.to(device) if device is not None else bt


class PagedKVLayerCache:
    def __init__(
        self,
        num_kv_heads: int,
        head_dim: int,
        max_seq_len: int,
        page_size: int,
        device: torch.device,
        dtype: torch.dtype,
        batch_size: int = 1,
        num_pages: int | None = None,
        block_table: torch.Tensor | None = None,
        workspace: DecodeWorkspace | None = None,
        status: torch.Tensor | None = None,
    ):
        if page_size <= 0:
            raise ValueError("page_size must be > 0")
        if max_seq_len <= 0:
            raise ValueError("max_seq_len must be > 0")
        if batch_size <= 0:
            raise ValueError("batch_size must be > 0")
        device = torch.device(device)
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.max_seq_len = max_seq_len
        self.page_size = page_size
        self.max_pages = math.ceil(max_seq_len / page_size)
        self.batch_size = batch_size
        self.device = device
        self.dtype = dtype
        if block_table is None:
            if num_pages is None:
                num_pages = batch_size * self.max_pages
            block_table = torch.arange(batch_size * self.max_pages, dtype=torch.int32).view(
                batch_size, self.max_pages)
        else:
            if block_table.shape != (batch_size, self.max_pages):
                raise ValueError("block_table must be [batch_size, ceil(max_seq_len / page_size)]")
            if num_pages is None:
                num_pages = int(block_table.max().item()) + 1
        self.num_pages = num_pages
        self.block_table = block_table.to(device=device, dtype=torch.int32).contiguous()
        self.key_pages = torch.empty(num_pages, num_kv_heads, page_size, head_dim, device=device,
                                     dtype=dtype)
        self.value_pages = torch.empty_like(self.key_pages)
        self.seq_lens = torch.zeros(batch_size, dtype=torch.int32, device=device)
        self.host_lengths = [0] * batch_size
        self.workspace = workspace if workspace is not None else DecodeWorkspace(device)
        self.status = status if status is not None else torch.zeros(1, dtype=torch.int32,
                                                                    device=device)

    # -- reference attributes ------------------------------------------------
    @property
    def length(self) -> int:
        """Tokens cached (the reference's ``length``); ragged batches have no single value."""
        first = self.host_lengths[0]
        if any(x != first for x in self.host_lengths):
            raise ValueError("ragged batch: per-sequence lengths are in host_lengths / seq_lens")
        return first

    # -- validation shared by the append paths --------------------------------
    def _check_kv(self, k: torch.Tensor, v: torch.Tensor) -> int:
        if k.shape != v.shape:
            raise ValueError("k and v shapes must match")
        if k.dim() != 4:
            raise ValueError("Expected k/v shape [batch, kv_heads, seq, head_dim]")
        if k.shape[0] != self.batch_size:
            raise ValueError(f"PagedKVLayerCache holds batch size {self.batch_size}")
        if k.shape[1] != self.num_kv_heads or k.shape[3] != self.head_dim:
            raise ValueError("k/v shapes do not match cache layout")
        seq = k.shape[2]
        if max(self.host_lengths) + seq > self.max_seq_len:
            raise ValueError("Appending would exceed max_seq_len")
        return seq

    def append(self, k: torch.Tensor, v: torch.Tensor) -> None:
        """Store already-rotated ``k`` and ``v`` ``[B, Hkv, S, d]`` (kv_cache.py:38-63)."""
        seq = self._check_kv(k, v)
        rope_append(None, k.to(self.dtype), v.to(self.dtype), self.key_pages, self.value_pages,
                    self.block_table, self.seq_lens, self.status)
        self.host_lengths = [x + seq for x in self.host_lengths]

    def append_rotary(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, rope: RopeTable,
                      q_out: torch.Tensor | None = None) -> torch.Tensor:
        """Fused RoPE + append: rotate raw ``q``/``k`` at each sequence's next positions,
        store k/v, return the rotated q (attention.py:110-123 in one launch)."""
        seq = self._check_kv(k, v)
        q_rot = rope_append(q, k, v, self.key_pages, self.value_pages, self.block_table,
                            self.seq_lens, self.status, cos=rope.cos, sin=rope.sin, q_out=q_out)
        self.host_lengths = [x + seq for x in self.host_lengths]
        return q_rot

    def rope_append_decode(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                           rope: RopeTable, out: torch.Tensor | None = None,
                           q_out: torch.Tensor | None = None,
                           partition_tokens: int | None = None,
                           early_tables: bool = False) -> torch.Tensor:
        """The whole decode-attention step of the new token: RoPE on q/k, page append
        and paged attention over the grown context, fused into one decode kernel (plus
        the merge).  Same results as ``append_rotary`` followed by ``decode``.
        ``early_tables``: see ``kernels.decode_attention.rope_append_decode``."""
        seq = self._check_kv(k, v)
        if seq != 1:
            raise ValueError("rope_append_decode takes one new token per sequence")
        res = rope_append_decode(q, k, v, self.key_pages, self.value_pages, self.block_table,
                                 self.seq_lens, rope.cos, rope.sin, host_lens=self.host_lengths,
                                 partition_tokens=partition_tokens, out=out, q_out=q_out,
                                 workspace=self.workspace, status=self.status,
                                 early_tables=early_tables)
        self.host_lengths = [x + 1 for x in self.host_lengths]
        return res

    def advance_host_lengths(self, n: int) -> None:
        """Mirror ``n`` appends replayed from a CUDA graph (the device already advanced)."""
        self.host_lengths = [x + n for x in self.host_lengths]

    def decode(self, q: torch.Tensor, out: torch.Tensor | None = None,
               partition_tokens: int | None = None) -> torch.Tensor:
        """Paged decode attention of ``q [B, Hq, 1, d]`` against this cache."""
        return paged_decode_attention(q, self, out=out, partition_tokens=partition_tokens)

    def get_kv(self) -> tuple[torch.Tensor, torch.Tensor]:
        """Gathered logical K/V ``[B, Hkv, len, d]`` (kv_cache.py:65-83); compatibility only."""
        L = self.length
        if L == 0:
            empty = self.key_pages.new_empty((self.batch_size, self.num_kv_heads, 0, self.head_dim))
            return empty, empty
        n = math.ceil(L / self.page_size)
        idx = self.block_table[:, :n].long()

        def gather(pages: torch.Tensor) -> torch.Tensor:
            g = pages[idx]                                    # [B, n, Hkv, P, d]
            g = g.permute(0, 2, 1, 3, 4).reshape(self.batch_size, self.num_kv_heads,
                                                 n * self.page_size, self.head_dim)
            return g[:, :, :L].contiguous()

        return gather(self.key_pages), gather(self.value_pages)

    def clear(self) -> None:
        self.seq_lens.zero_()
        self.host_lengths = [0] * self.batch_size

    def check_status(self) -> None:
        """Synchronise and raise ``DeviceStatusError`` if a kernel flagged an error."""
        try:
            N.raise_on_status(self.status)
        except N.DeviceStatusError:
            self.workspace.invalidate_counters()
            raise


class PagedKVCache:
    def __init__(self, layer_caches: list[PagedKVLayerCache]):
        if not layer_caches:
            raise ValueError("layer_caches must not be empty")
        self.layer_caches = layer_caches

    @classmethod
    def create(
        cls,
        num_layers: int,
        num_kv_heads: int,
        head_dim: int,
        max_seq_len: int,
        page_size: int,
        device: torch.device,
        dtype: torch.dtype,
        batch_size: int = 1,
        num_pages: int | None = None,
        block_table: torch.Tensor | None = None,
    ) -> "PagedKVCache":
        """One layer cache per layer; all layers share the block table, the split-K
        workspace and the status word (each layer has its own page pools and lengths)."""
        device = torch.device(device)
        ws = DecodeWorkspace(device)
        status = torch.zeros(1, dtype=torch.int32, device=device)
        return cls([
            PagedKVLayerCache(num_kv_heads=num_kv_heads, head_dim=head_dim,
                              max_seq_len=max_seq_len, page_size=page_size, device=device,
                              dtype=dtype, batch_size=batch_size, num_pages=num_pages,
                              block_table=block_table, workspace=ws, status=status)
            for _ in range(num_layers)
        ])

    def get_layer(self, layer_idx: int) -> PagedKVLayerCache:
        return self.layer_caches[layer_idx]

    def clear(self) -> None:
        for layer in self.layer_caches:
            layer.clear()

    def check_status(self) -> None:
        self.layer_caches[0].check_status()


class GraphedDecodeStep:
    """The fused decode-attention step of one cache, captured once as a CUDA graph.

    ``q``/``k``/``v`` are device input buffers (``[B, Hq|Hkv, 1, d]``) that the caller
    refills before each ``replay()``; the step rotates, appends at ``seq_lens`` and
    attends, advancing the lengths on the device and in ``cache.host_lengths``.  One
    graph launch per step instead of several Python-issued launches: the host cost of
    a step is that of ``cudaGraphLaunch``.  By default the step uses the balanced
    split, which the kernel recomputes from the device lengths at every replay, so
    the work stays even across SMs as the contexts grow.
    """

    def __init__(self, cache: PagedKVLayerCache, rope: RopeTable, q: torch.Tensor,
                 k: torch.Tensor, v: torch.Tensor, partition_tokens: int | None = None,
                 out: torch.Tensor | None = None):
        from ...kernels.decode_attention import BALANCED

        self.cache, self.rope, self.q, self.k, self.v = cache, rope, q, k, v
        B, Hq, d = q.shape[0], q.shape[1], q.shape[-1]
        self.partition_tokens = BALANCED if partition_tokens is None else partition_tokens
        self.out = out if out is not None else torch.empty(B, Hq, d, dtype=q.dtype,
                                                           device=q.device)
        self.q_rot = torch.empty(B, Hq, d, dtype=q.dtype, device=q.device)
        lens0 = cache.seq_lens.clone()
        host0 = list(cache.host_lengths)
        self._step()                          # warm-up: workspaces exist before capture
        torch.cuda.synchronize(q.device)
        cache.seq_lens.copy_(lens0)
        s = torch.cuda.Stream(device=q.device)
        s.wait_stream(torch.cuda.current_stream(q.device))
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(self.graph, stream=s):
                self._step()
        torch.cuda.current_stream(q.device).wait_stream(s)
        torch.cuda.synchronize(q.device)
        cache.seq_lens.copy_(lens0)
        cache.host_lengths = host0

    def _step(self):
        c = self.cache
        rope_append_decode(self.q, self.k, self.v, c.key_pages, c.value_pages, c.block_table,
                           c.seq_lens, self.rope.cos, self.rope.sin,
                           partition_tokens=self.partition_tokens, out=self.out,
                           q_out=self.q_rot, workspace=c.workspace, status=c.status)

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        self.cache.advance_host_lengths(1)
        return self.out
