"""Pin the CPU oracle to the reference's own outputs (golden fixtures).

The fixtures were produced by running llm-cuda's CPU path
(``tests/golden/make_golden.py``); inputs are regenerated from seeds and checked
against the SHA-256 recorded in each fixture.
"""

import os

import numpy as np
import pytest
import torch

import cases as C
from oracle import decode_oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _load(name):
    return np.load(os.path.join(GOLD, name))


def _f(t: torch.Tensor, dt: str) -> np.ndarray:
    return O.from_bits(C.to_np(t), dt)


def assert_ulp_close(out, ref, dt, min_exact=0.99):
    """16-bit results: within one unit in the last place (1e-4 absolute near zero,
    where a cancelling fp32 sum meets a different accumulation
    order) and bit-exact almost everywhere."""
    rtol = {"bf16": 2.0 ** -7, "fp16": 2.0 ** -10}[dt]
    np.testing.assert_allclose(out, ref, rtol=rtol, atol=1e-4)
    assert np.mean(out == ref) >= min_exact


def test_round_to_bf16_matches_torch():
    x = torch.randn(10000) * 100
    x[:4] = torch.tensor([0.0, -0.0, 1e-40, 65504.0])
    ours = O.round_to(x.numpy(), "bf16")
    ref = x.to(torch.bfloat16).float().numpy()
    assert np.array_equal(ours, ref)
    assert np.array_equal(O.round_to(x.numpy(), "fp16"), x.to(torch.float16).float().numpy())


@pytest.mark.parametrize("name", list(C.DENSE_CASES))
def test_oracle_dense_cases(name):
    g = _load("dense_cases.npz")
    B, Hq, Hkv, L, d, dt = C.DENSE_CASES[name]
    q, k, v = C.dense_inputs(name)
    assert str(g[f"{name}__sha"]) == C.sha(q, k, v), "regenerated inputs differ from the fixture's"
    qn, kn, vn = _f(q, dt), _f(k, dt), _f(v, dt)
    out = np.stack([O.decode_attention(qn[b, :, 0], kn[b], vn[b], dt) for b in range(B)])
    ref = O.from_bits(g[f"{name}__out"], dt)[:, :, 0]
    if dt == "fp32":
        np.testing.assert_allclose(out, ref, rtol=1e-5, atol=1e-6)
    else:  # 16-bit: restatement of the reference's rounding points
        assert_ulp_close(out, ref, dt)


@pytest.mark.parametrize("dt", list(C.ROPE_CASES))
def test_oracle_rope(dt):
    r = _load("rope_cases.npz")
    d, H = C.ROPE_CASES[dt]
    x = C.rope_inputs(dt)
    assert str(r[f"{dt}__sha"]) == C.sha(x)
    np.testing.assert_array_equal(O.build_inv_freq(d, C.THETA), r[f"{dt}__inv_freq"])
    cos, sin = O.build_rope_cache(C.ROPE_POSITIONS, d, C.THETA, dt)
    rc, rs = O.from_bits(r[f"{dt}__cos"], dt), O.from_bits(r[f"{dt}__sin"], dt)
    if dt == "fp32":  # numpy vs torch fp32 cos/sin may differ by one ulp
        np.testing.assert_allclose(cos, rc, rtol=0, atol=1.2e-7)
        np.testing.assert_allclose(sin, rs, rtol=0, atol=1.2e-7)
    else:
        np.testing.assert_array_equal(cos, rc)
        np.testing.assert_array_equal(sin, rs)
    xf = _f(x, dt)
    out = np.stack([O.apply_rotary(xf[i], cos[i:i + 1], sin[i:i + 1], dt)
                    for i in range(len(C.ROPE_POSITIONS))])
    ref = O.from_bits(r[f"{dt}__out"], dt)
    if dt == "fp32":
        np.testing.assert_allclose(out, ref, rtol=0, atol=1e-6)
    else:
        np.testing.assert_array_equal(out, ref)


@pytest.mark.parametrize("name", list(C.STEP_CASES))
def test_oracle_decode_step(name):
    """RoPE + append into a shuffled page pool + attend, against the reference."""
    g = _load(f"step_{name}.npz")
    dt, Hq, Hkv, d, lens, scale, seed = C.STEP_CASES[name]
    seqs = C.step_inputs(name)
    flat = [t for s in seqs for t in s]
    assert str(g["input_sha"]) == C.sha(*flat)
    P = 16
    B = len(lens)
    max_pages = max((L + P - 1) // P for L in lens)
    rng = np.random.default_rng(seed)
    num_pages = B * max_pages + 3
    perm = rng.permutation(num_pages)
    bt = perm[:B * max_pages].reshape(B, max_pages)
    kp = np.full((num_pages, Hkv, P, d), np.nan, np.float32)   # untouched slots are NaN
    vp = np.full_like(kp, np.nan)
    for b, (pk, pv, *_rest) in enumerate(seqs):
        O.append_tokens(kp, bt[b], 0, _f(pk, dt))
        O.append_tokens(vp, bt[b], 0, _f(pv, dt))
    cos, sin = O.build_rope_cache(np.arange(max(lens)), d, C.THETA, dt)
    q_raw = np.stack([_f(s[2], dt) for s in seqs])
    k_raw = np.stack([_f(s[3], dt) for s in seqs])
    v_raw = np.stack([_f(s[4], dt) for s in seqs])
    q_rot, out, new_lens = O.decode_step(kp, vp, bt, np.array(lens) - 1, q_raw, k_raw, v_raw,
                                         cos, sin, dt)
    assert list(new_lens) == lens
    ref_out = O.from_bits(g["out"], dt)
    if dt == "fp32":
        np.testing.assert_allclose(q_rot, O.from_bits(g["q_rot"], dt), rtol=0, atol=1e-6)
        np.testing.assert_allclose(out, ref_out, rtol=1e-5, atol=1e-6)
    else:
        np.testing.assert_array_equal(q_rot, O.from_bits(g["q_rot"], dt))
        assert_ulp_close(out, ref_out, dt)


def test_oracle_c1_sequence():
    """Config 1 end to end: 64-token prefill then 16 decode steps, permuted 8-page pool."""
    g = _load("c1_fp32.npz")
    q, k, v, perm = C.c1_inputs()
    assert str(g["input_sha"]) == C.sha(q, k, v, perm)
    q, k, v = q.numpy()[0], k.numpy()[0], v.numpy()[0]
    P, d = 64, q.shape[-1]
    bt = perm.numpy()[:2][None]                   # 80 tokens -> 2 pages of the pool
    kp = np.zeros((8, 2, P, d), np.float32)
    vp = np.zeros_like(kp)
    cos, sin = O.build_rope_cache(np.arange(80), d, C.THETA, "fp32")
    k_rot = O.apply_rotary(k[:, :64], cos[:64], sin[:64], "fp32")
    O.append_tokens(kp, bt[0], 0, k_rot)
    O.append_tokens(vp, bt[0], 0, v[:, :64])
    lens = np.array([64])
    outs = []
    for t in range(16):
        i = 64 + t
        _, out, lens = O.decode_step(kp, vp, bt, lens, q[None, :, i], k[None, :, i], v[None, :, i],
                                     cos, sin, "fp32")
        outs.append(out[0])
    ref = g["out"][:, 0, :, 0]
    np.testing.assert_allclose(np.stack(outs), ref, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(O.gather_logical(kp, bt[0], 80), g["k_cache"][0], rtol=0, atol=1e-6)
