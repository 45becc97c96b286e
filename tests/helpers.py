"""Test-side helpers: build paged caches from logical K/V and compare with the oracle."""

from __future__ import annotations

import numpy as np
import torch

import cases as C
from oracle import decode_oracle as O

NAMES = {torch.float32: "fp32", torch.float16: "fp16", torch.bfloat16: "bf16"}

# Parity bars (north star): fp32 1e-5 relative, bf16 2e-2 absolute; fp16 follows the
# reference's own fp16 test tolerance (tests/test_triton_decode_attention.py:214-226).
TOL = {"fp32": dict(rtol=1e-5, atol=1e-6), "bf16": dict(rtol=0.0, atol=2e-2),
       "fp16": dict(rtol=0.0, atol=1e-2)}


def to_f32_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def fill_pages(cache, ks, vs):
    """Write per-sequence logical K/V (``[Hkv, L_b, d]`` tensors) into a cache's pages
    through its block table and set its lengths (host-side test set-up)."""
    P = cache.page_size
    bt = cache.block_table.cpu()
    for b, (k, v) in enumerate(zip(ks, vs)):
        L = k.shape[1]
        if L == 0:
            continue
        n = (L + P - 1) // P
        pad = n * P - L
        kk = torch.nn.functional.pad(k, (0, 0, 0, pad)).view(k.shape[0], n, P, k.shape[2])
        vv = torch.nn.functional.pad(v, (0, 0, 0, pad)).view(v.shape[0], n, P, v.shape[2])
        pages = bt[b, :n].long().to(cache.device)
        # keep whatever the padding slots held before (they must never be read)
        kold = cache.key_pages[pages].clone()
        vold = cache.value_pages[pages].clone()
        knew = kk.permute(1, 0, 2, 3).to(cache.device, cache.dtype)
        vnew = vv.permute(1, 0, 2, 3).to(cache.device, cache.dtype)
        knew[-1, :, P - pad:] = kold[-1, :, P - pad:]
        vnew[-1, :, P - pad:] = vold[-1, :, P - pad:]
        cache.key_pages[pages] = knew
        cache.value_pages[pages] = vnew
    lens = [k.shape[1] for k in ks]
    cache.seq_lens.copy_(torch.tensor(lens, dtype=torch.int32))
    cache.host_lengths = list(lens)


def poison(cache, value=float("nan")):
    """Fill every page slot with NaN so that any read past a context shows up."""
    cache.key_pages.fill_(value)
    cache.value_pages.fill_(value)


def oracle_decode(q: torch.Tensor, ks, vs) -> np.ndarray:
    """Oracle attention for ``q [B, Hq, d]`` and per-sequence logical K/V."""
    dt = NAMES[q.dtype]
    qn = to_f32_np(q)
    return np.stack([O.decode_attention(qn[b], to_f32_np(ks[b]), to_f32_np(vs[b]), dt)
                     for b in range(len(ks))])


def assert_parity(out: torch.Tensor, ref: np.ndarray, dtype: torch.dtype, what: str = ""):
    tol = TOL[NAMES[dtype]]
    got = to_f32_np(out).reshape(ref.shape)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    np.testing.assert_allclose(got, ref, err_msg=what, **tol)
