"""CPU oracle for the decode-attention path — TEST INFRASTRUCTURE ONLY.

A numpy restatement of calvin-fei/llm-cuda's CPU decode path, used only as the
checker by ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline leg.  Nothing in the product package imports this module: the product
path runs the CUDA kernels in ``llm_cuda_b200/csrc`` and fails loudly if they are
missing.

Parity is pinned: ``tests/test_oracle_golden.py`` checks every function here
against fixtures produced by running the reference itself
(``tests/golden/make_golden.py``).

What is restated (paths inside the llm-cuda project):

* ``build_inv_freq``      — ``src/llm_cuda/models/llama3/rotary.py:6-26``
* ``build_rope_cache``    — ``src/llm_cuda/models/llama3/rotary.py:29-71``
* ``apply_rotary``        — ``src/llm_cuda/models/llama3/rotary.py:74-78,104-109``
  (the torch fallback: every product and the sum are rounded to the tensor dtype)
* ``gather_logical``      — ``src/llm_cuda/models/llama3/kv_cache.py:65-83``
  (``get_kv``), generalised to a block table over a shared page pool
* ``decode_attention``    — ``src/llm_cuda/models/llama3/attention.py:56-89``
  (``_repeat_kv`` + ``_torch_attention``: matmul rounded to dtype, ``/ sqrt(d)``
  rounded, causal mask, softmax computed in fp32 and rounded, matmul rounded)

16-bit floating types are emulated on float32 arrays holding exactly
representable values; ``round_to`` rounds to nearest-even like torch's casts.
"""

from __future__ import annotations

import numpy as np

FP32, BF16, FP16 = "fp32", "bf16", "fp16"


# ---------------------------------------------------------------------------
# dtype emulation
# ---------------------------------------------------------------------------

def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` (round-to-nearest-even), returned as float32."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == FP32:
        return x
    if dtype == FP16:
        return x.astype(np.float16).astype(np.float32)
    if dtype == BF16:
        b = x.view(np.uint32).astype(np.uint64)
        nan = np.isnan(x)
        b = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000
        out = b.astype(np.uint32).view(np.float32)
        return np.where(nan, np.float32(np.nan), out).astype(np.float32)
    raise ValueError(f"unknown dtype {dtype}")


def from_bits(bits: np.ndarray, dtype: str) -> np.ndarray:
    """Decode stored fixture values (uint16 bit patterns for 16-bit types) to float32."""
    if dtype == FP32:
        return np.asarray(bits, dtype=np.float32)
    bits = np.asarray(bits, dtype=np.uint16)
    if dtype == FP16:
        return bits.view(np.float16).astype(np.float32)
    return (bits.astype(np.uint32) << 16).view(np.float32)


def to_bits(x: np.ndarray, dtype: str) -> np.ndarray:
    """Encode float32 values (already representable in ``dtype``) as fixture values."""
    x = round_to(x, dtype)
    if dtype == FP32:
        return x
    if dtype == FP16:
        return x.astype(np.float16).view(np.uint16)
    return (x.view(np.uint32) >> 16).astype(np.uint16)


# ---------------------------------------------------------------------------
# RoPE  (rotary.py)
# ---------------------------------------------------------------------------

def build_inv_freq(head_dim: int, base: float) -> np.ndarray:
    """``1 / base ** (arange(0, d, 2) / d)`` in float32 (rotary.py:24-26).

    The exponent is the fp32 quotient; the power is the correctly rounded fp32 value
    (computed in fp64, then rounded), which is what torch returns for this op and
    what the golden ``inv_freq`` vectors hold bit for bit."""
    expo = np.arange(0, head_dim, 2, dtype=np.float32) / np.float32(head_dim)
    powed = np.power(np.float64(base), expo.astype(np.float64)).astype(np.float32)
    return (np.float32(1.0) / powed).astype(np.float32)


def build_rope_cache(positions, head_dim: int, base: float, dtype: str):
    """cos/sin ``[len(positions), head_dim]`` (rotary.py:54-71): fp32 outer product of
    positions and inv_freq, duplicated halves, cos/sin in fp32, rounded to ``dtype``."""
    pos = np.asarray(positions, dtype=np.float32)
    freqs = np.outer(pos, build_inv_freq(head_dim, base)).astype(np.float32)
    emb = np.concatenate([freqs, freqs], axis=-1)
    return round_to(np.cos(emb), dtype), round_to(np.sin(emb), dtype)


def rotate_half(x: np.ndarray) -> np.ndarray:
    """rotary.py:74-78."""
    h = x.shape[-1] // 2
    return np.concatenate([-x[..., h:], x[..., :h]], axis=-1)


def apply_rotary(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, dtype: str) -> np.ndarray:
    """``x * cos + rotate_half(x) * sin`` with torch's per-op rounding (rotary.py:104-109).

    ``x`` is ``[..., S, d]``; ``cos``/``sin`` are ``[S, d]`` broadcast over the leading dims.
    """
    a = round_to(x * cos, dtype)
    b = round_to(rotate_half(x) * sin, dtype)
    return round_to(a + b, dtype)


# ---------------------------------------------------------------------------
# Paged KV  (kv_cache.py)
# ---------------------------------------------------------------------------

def gather_logical(pages: np.ndarray, block_row: np.ndarray, length: int) -> np.ndarray:
    """Logical ``[Hkv, length, d]`` of one sequence from ``pages[num_pages, Hkv, P, d]``.

    The reference stores token ``t`` at page ``t // P``, slot ``t % P``
    (kv_cache.py:55-61) and gathers pages in order (kv_cache.py:65-83); with a
    block table the physical page is ``block_row[t // P]``.
    """
    P = pages.shape[2]
    n = (length + P - 1) // P
    if n == 0:
        return np.zeros((pages.shape[1], 0, pages.shape[3]), dtype=pages.dtype)
    chunks = pages[np.asarray(block_row[:n], dtype=np.int64)]          # [n, Hkv, P, d]
    full = np.transpose(chunks, (1, 0, 2, 3)).reshape(pages.shape[1], n * P, pages.shape[3])
    return full[:, :length]


def append_tokens(pages: np.ndarray, block_row: np.ndarray, start: int, kv_new: np.ndarray) -> None:
    """Write ``kv_new[Hkv, S, d]`` at positions ``start .. start+S-1`` (kv_cache.py:55-61)."""
    P = pages.shape[2]
    for s in range(kv_new.shape[1]):
        t = start + s
        pages[int(block_row[t // P]), :, t % P, :] = kv_new[:, s, :]


# ---------------------------------------------------------------------------
# Attention  (attention.py:56-89)
# ---------------------------------------------------------------------------

def decode_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, dtype: str) -> np.ndarray:
    """One sequence, one query token at position ``L-1`` attending to ``L`` cached tokens.

    ``q[Hq, d]``, ``k``/``v`` ``[Hkv, L, d]`` → ``[Hq, d]``.  Query head ``h`` reads KV
    head ``h // (Hq // Hkv)`` (``_repeat_kv``, attention.py:56-61).  The causal mask of
    ``_torch_attention`` (attention.py:75-83) admits every cached position for a
    decode query, so it adds zero.  Each torch op's rounding to ``dtype`` is kept:
    scores (matmul, then ``/ sqrt(d)``), probabilities (fp32 softmax, rounded) and
    the output (matmul).
    """
    Hq, d = q.shape
    Hkv, L, _ = k.shape
    out = np.zeros((Hq, d), dtype=np.float32)
    if L == 0:
        return out
    G = Hq // Hkv
    inv = np.float32(1.0) / np.float32(np.sqrt(np.float64(d)))
    for kvh in range(Hkv):
        qg = q[kvh * G:(kvh + 1) * G].astype(np.float32)                   # [G, d]
        s = round_to(qg @ k[kvh].astype(np.float32).T, dtype)               # [G, L]
        s = round_to(s * inv, dtype) if dtype != FP32 else (s / np.float32(np.sqrt(d))).astype(np.float32)
        m = s.max(axis=-1, keepdims=True)
        e = np.exp((s - m).astype(np.float32)).astype(np.float32)
        p = round_to(e / e.sum(axis=-1, keepdims=True, dtype=np.float32), dtype)
        out[kvh * G:(kvh + 1) * G] = round_to(p @ v[kvh].astype(np.float32), dtype)
    return out


def decode_step(pages_k, pages_v, block_table, seq_lens, q_raw, k_raw, v_raw, cos_tab, sin_tab, dtype):
    """The whole hot path for a batch, one decode token per sequence.

    For each sequence ``b`` at position ``pos = seq_lens[b]``: RoPE on the new q and k
    (rotary.py:104-109, table rows ``pos``), append k/v at ``pos`` (kv_cache.py:55-61),
    then attend over ``pos + 1`` tokens (attention.py:56-89).  Mutates the page pools
    and returns ``(q_rot[B,Hq,d], out[B,Hq,d], new_seq_lens)``.
    """
    B = q_raw.shape[0]
    q_rot = np.zeros_like(q_raw, dtype=np.float32)
    out = np.zeros_like(q_raw, dtype=np.float32)
    new_lens = np.asarray(seq_lens).copy()
    for b in range(B):
        pos = int(seq_lens[b])
        cos, sin = cos_tab[pos:pos + 1], sin_tab[pos:pos + 1]
        q_rot[b] = apply_rotary(q_raw[b][:, None], cos, sin, dtype)[:, 0]
        k_rot = apply_rotary(k_raw[b][:, None], cos, sin, dtype)
        append_tokens(pages_k, block_table[b], pos, k_rot)
        append_tokens(pages_v, block_table[b], pos, v_raw[b][:, None])
        L = pos + 1
        new_lens[b] = L
        out[b] = decode_attention(q_rot[b], gather_logical(pages_k, block_table[b], L),
                                  gather_logical(pages_v, block_table[b], L), dtype)
    return q_rot, out, new_lens
