"""RoPE tables with the reference's numerics, and the fused RoPE+append entry.

``build_inv_freq`` / ``build_rope_cache`` keep the reference's signatures and
arithmetic (``src/llm_cuda/models/llama3/rotary.py:6-71`` of llm-cuda): fp32
``inv_freq``, fp32 outer product with the positions, ``cat(freqs, freqs)``,
``cos``/``sin`` in fp32, cast to the model dtype.  They are evaluated on the CPU
once per cache (the table covers every position the cache can hold), so the
decode step never rebuilds them (the reference rebuilds them per layer per step,
attention.py:110-118) and the values are bit-identical to the reference's CPU
tables.  The rotation itself runs inside the fused CUDA kernel
(``llm_cuda_b200.kernels.rope``).
"""

from __future__ import annotations

import torch


def build_inv_freq(head_dim: int, base: float, device: torch.device) -> torch.Tensor:
    """``1 / base ** (arange(0, d, 2) / d)`` as float32 ``[head_dim // 2]``."""
    return 1.0 / (base ** (torch.arange(0, head_dim, 2, device=device, dtype=torch.float32) / head_dim))


def build_rope_cache(
    seq_len: int,
    head_dim: int,
    base: float,
    device: torch.device,
    dtype: torch.dtype,
    position_offset: int = 0,
    inv_freq: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin ``[seq_len, head_dim]`` for positions ``position_offset ..``."""
    if inv_freq is None:
        inv_freq = build_inv_freq(head_dim, base, device)
    elif inv_freq.device != device:
        inv_freq = inv_freq.to(device=device)
    positions = torch.arange(position_offset, position_offset + seq_len, device=device,
                             dtype=torch.float32)
    freqs = torch.outer(positions, inv_freq)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype=dtype), emb.sin().to(dtype=dtype)


class RopeTable:
    """Device-resident cos/sin rows for positions ``0 .. max_positions-1``.

    Built on the CPU with :func:`build_rope_cache` (bit-identical to the reference's
    CPU tables) and copied to ``device`` once.
    """

    def __init__(self, max_positions: int, head_dim: int, base: float, device, dtype):
        cos, sin = build_rope_cache(max_positions, head_dim, base, torch.device("cpu"), dtype)
        self.cos = cos.to(device).contiguous()
        self.sin = sin.to(device).contiguous()
        self.max_positions = max_positions
        self.head_dim = head_dim
        self.base = base
