"""Seeded input generators shared by the fixture generator and the tests.

Inputs are regenerated from ``torch.Generator`` seeds (the CPU generator is
deterministic for a given torch build) instead of being stored, which keeps the
fixtures small.  Each fixture records a SHA-256 of the inputs it was made from,
so a test that regenerates different inputs fails loudly instead of comparing
against the wrong golden output.
"""

from __future__ import annotations

import hashlib

import numpy as np
import torch

DTYPES = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}
THETA = 500000.0

# Single decode steps (RoPE on the new token, append, attend) over ragged batches.
# name: (dtype, Hq, Hkv, d, lengths after the append, value scale, seed)
STEP_CASES = {
    "llama8b_bf16": ("bf16", 32, 8, 128, [300, 77], 1.0, 1002),
    "ragged_edges_bf16": ("bf16", 32, 8, 128, [1, 15, 16, 17, 64, 65, 129], 1.0, 1003),
    "llama70b_bf16": ("bf16", 64, 8, 128, [5000], 0.5, 1004),
    "gqa_fp16": ("fp16", 16, 8, 64, [128, 3], 1.0, 1005),
    "gqa_fp32": ("fp32", 8, 2, 64, [200, 1, 64], 1.0, 1006),
}

# The reference kernel test shapes (tests/test_triton_decode_attention.py:177-303),
# dense K/V, seed 42: name: (B, Hq, Hkv, L, d, dtype)
DENSE_CASES = {
    "mha_fp32": (2, 4, 4, 64, 32, "fp32"),
    "gqa_fp32": (2, 8, 4, 64, 32, "fp32"),
    "gqa_fp16": (1, 16, 8, 128, 64, "fp16"),
    "gqa_bf16": (1, 16, 8, 128, 64, "bf16"),
    "single_kv": (1, 4, 2, 1, 16, "fp32"),
    "long_kv": (1, 8, 4, 1024, 64, "fp32"),
    "hd48": (1, 4, 2, 32, 48, "fp32"),
    "batch4": (4, 8, 4, 64, 32, "fp32"),
}

# RoPE on single tokens at scattered positions: dtype: (head_dim, heads)
ROPE_CASES = {"fp32": (64, 4), "bf16": (128, 8), "fp16": (128, 2)}
ROPE_POSITIONS = [0, 1, 15, 16, 4095, 32767, 131071]


def sha(*tensors: torch.Tensor) -> str:
    h = hashlib.sha256()
    for t in tensors:
        t = t.detach().cpu().contiguous()
        if t.dtype in (torch.bfloat16, torch.float16):
            t = t.view(torch.int16)
        h.update(t.numpy().tobytes())
    return h.hexdigest()


def c1_inputs():
    """Config 1: fp32, B1 Hq8 Hkv2 d64, 64 prompt + 16 decode tokens, page 64,
    an 8-page pool in random order.  Returns raw (pre-RoPE) q/k/v over all 80
    positions and the pool permutation."""
    g = torch.Generator().manual_seed(1001)
    Hq, Hkv, d, total = 8, 2, 64, 80
    q = torch.randn(1, Hq, total, d, generator=g)
    k = torch.randn(1, Hkv, total, d, generator=g)
    v = torch.randn(1, Hkv, total, d, generator=g)
    perm = torch.randperm(8, generator=g).to(torch.int32)
    return q, k, v, perm


def step_inputs(name: str):
    """Per sequence: cached K/V (``[Hkv, L-1, d]``, stored as-is) and the new
    token's raw q ``[Hq, d]``, k and v ``[Hkv, d]``."""
    dt, Hq, Hkv, d, lens, scale, seed = STEP_CASES[name]
    dtype = DTYPES[dt]
    g = torch.Generator().manual_seed(seed)
    seqs = []
    for L in lens:
        pk = (torch.randn(1, Hkv, L - 1, d, generator=g) * scale).to(dtype)
        pv = (torch.randn(1, Hkv, L - 1, d, generator=g) * scale).to(dtype)
        qn = (torch.randn(1, Hq, 1, d, generator=g) * scale).to(dtype)
        kn = (torch.randn(1, Hkv, 1, d, generator=g) * scale).to(dtype)
        vn = (torch.randn(1, Hkv, 1, d, generator=g) * scale).to(dtype)
        seqs.append((pk[0], pv[0], qn[0, :, 0], kn[0, :, 0], vn[0, :, 0]))
    return seqs


def dense_inputs(name: str):
    B, Hq, Hkv, L, d, dt = DENSE_CASES[name]
    dtype = DTYPES[dt]
    torch.manual_seed(42)
    q = torch.randn(B, Hq, 1, d, dtype=dtype)
    k = torch.randn(B, Hkv, L, d, dtype=dtype)
    v = torch.randn(B, Hkv, L, d, dtype=dtype)
    return q, k, v


def rope_inputs(dt: str):
    d, H = ROPE_CASES[dt]
    g = torch.Generator().manual_seed(99)
    return torch.randn(len(ROPE_POSITIONS), H, 1, d, generator=g).to(DTYPES[dt])


def to_torch(a: np.ndarray, dt: str) -> torch.Tensor:
    """Inverse of the fixture encoding: 16-bit types are stored as uint16 bits."""
    if dt == "fp32":
        return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(DTYPES[dt])


def to_np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()
