"""Generate the golden fixtures under ``tests/golden/`` by running the REFERENCE.

This script is the only file in the repository that imports calvin-fei/llm-cuda.
It runs the reference's own CPU code path for decode attention on small seeded
inputs and stores inputs and outputs as ``.npz`` files.  The fixtures travel with
the repository; the reference tree does not (tests never import it).

Reference functions exercised (paths inside the llm-cuda project):

* ``src/llm_cuda/models/llama3/rotary.py:6-26``   build_inv_freq
* ``src/llm_cuda/models/llama3/rotary.py:29-71``  build_rope_cache
* ``src/llm_cuda/models/llama3/rotary.py:81-109`` apply_rotary (torch fallback on CPU)
* ``src/llm_cuda/models/llama3/kv_cache.py:38-83`` PagedKVLayerCache.append / get_kv
* ``src/llm_cuda/models/llama3/attention.py:56-89`` _repeat_kv + _torch_attention
* ``src/llm_cuda/models/llama3/model.py:110-218`` Llama3ForCausalLM (tiny decode parity)

Usage (in a container that has the reference checked out)::

    python tests/golden/make_golden.py --ref-src <llm-cuda>/src

Inputs are regenerated from seeds by ``cases.py``; fixtures store outputs and a
SHA-256 of the inputs.  bf16/fp16 tensors are stored as raw 16-bit patterns
(``uint16``) so the
fixtures are bit-exact; fp32 tensors are stored as ``float32``.
"""

from __future__ import annotations

import argparse
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

sys.path.insert(0, HERE)
import cases as C  # noqa: E402


def _attn_self(num_heads: int, num_kv_heads: int, head_dim: int):
    """A stand-in ``self`` for the reference's unbound attention helpers."""
    return types.SimpleNamespace(
        num_heads=num_heads,
        num_kv_heads=num_kv_heads,
        head_dim=head_dim,
        num_kv_groups=num_heads // num_kv_heads,
    )


def _ref_decode(ref, q, k, v, past_len):
    """reference ``_repeat_kv`` + ``_torch_attention`` (attention.py:56-89)."""
    Attn = ref["Llama3Attention"]
    s = _attn_self(q.shape[1], k.shape[1], q.shape[-1])
    kk = Attn._repeat_kv(s, k)
    vv = Attn._repeat_kv(s, v)
    return Attn._torch_attention(s, q, kk, vv, attention_mask=None, past_len=past_len)


def _ref_step(ref, q_raw, k_raw, v_raw, cache, dtype):
    """One reference decode step for one sequence (attention.py:104-147)."""
    pos = cache.length
    head_dim = q_raw.shape[-1]
    inv = ref["build_inv_freq"](head_dim, C.THETA, torch.device("cpu"))
    cos, sin = ref["build_rope_cache"](
        seq_len=q_raw.shape[-2], head_dim=head_dim, base=C.THETA, device=torch.device("cpu"),
        dtype=dtype, position_offset=pos, inv_freq=inv)
    q, k = ref["apply_rotary"](q_raw, k_raw, cos, sin)
    cache.append(k, v_raw)
    kc, vc = cache.get_kv()
    out = _ref_decode(ref, q, kc, vc, past_len=pos)
    return q, k, out


def gen_c1(ref):
    """Config 1: fp32, B1 Hq8 Hkv2 d64, 64 prompt tokens then 16 decode steps, P=64."""
    q_all, k_all, v_all, perm = C.c1_inputs()
    Hkv, d = k_all.shape[1], k_all.shape[-1]
    prompt, steps, P = 64, 16, 64
    total = prompt + steps
    cache = ref["PagedKVLayerCache"](Hkv, d, total, P, torch.device("cpu"), torch.float32)
    # Prefill: RoPE at positions 0..63, then append (attention.py:110-123).
    inv = ref["build_inv_freq"](d, C.THETA, torch.device("cpu"))
    cos, sin = ref["build_rope_cache"](prompt, d, C.THETA, torch.device("cpu"), torch.float32, 0, inv)
    _, k_rot = ref["apply_rotary"](q_all[:, :, :prompt], k_all[:, :, :prompt], cos, sin)
    cache.append(k_rot, v_all[:, :, :prompt])
    outs, qrots = [], []
    for t in range(steps):
        i = prompt + t
        q, _, out = _ref_step(ref, q_all[:, :, i:i + 1], k_all[:, :, i:i + 1],
                              v_all[:, :, i:i + 1], cache, torch.float32)
        outs.append(out)
        qrots.append(q)
    kc, vc = cache.get_kv()
    np.savez_compressed(
        os.path.join(HERE, "c1_fp32.npz"), input_sha=C.sha(q_all, k_all, v_all, perm),
        prompt=prompt, steps=steps, page_size=P,
        out=C.to_np(torch.stack(outs)), q_rot=C.to_np(torch.stack(qrots)),
        k_cache=C.to_np(kc), v_cache=C.to_np(vc))


def gen_step_cases(ref):
    """Single decode steps (RoPE + append + attend) on ragged batches, one sequence
    at a time through the reference (its cache is batch-1 only, kv_cache.py:43-44)."""
    for name, (dt, Hq, Hkv, d, lens, scale, seed) in C.STEP_CASES.items():
        dtype = C.DTYPES[dt]
        seqs = C.step_inputs(name)
        q_rot, k_rot, outs = [], [], []
        flat = []
        for L, (pk, pv, qn, kn, vn) in zip(lens, seqs):
            cache = ref["PagedKVLayerCache"](Hkv, d, L, 16, torch.device("cpu"), dtype)
            if L > 1:
                cache.append(pk[None], pv[None])  # cached tokens are stored as-is
            q, k, out = _ref_step(ref, qn[None, :, None], kn[None, :, None], vn[None, :, None],
                                  cache, dtype)
            q_rot.append(C.to_np(q[0, :, 0]))
            k_rot.append(C.to_np(k[0, :, 0]))
            outs.append(C.to_np(out[0, :, 0]))
            flat += [pk, pv, qn, kn, vn]
        np.savez_compressed(
            os.path.join(HERE, f"step_{name}.npz"), input_sha=C.sha(*flat),
            q_rot=np.stack(q_rot), k_rot=np.stack(k_rot), out=np.stack(outs))


def gen_dense_cases(ref):
    """The reference kernel test shapes (tests/test_triton_decode_attention.py:177-303),
    seed 42, dense K/V, outputs from the reference torch path."""
    arrays = {}
    for name in C.DENSE_CASES:
        q, k, v = C.dense_inputs(name)
        out = _ref_decode(ref, q, k, v, past_len=k.shape[2] - 1)
        arrays[f"{name}__out"] = C.to_np(out)
        arrays[f"{name}__sha"] = np.array(C.sha(q, k, v))
    np.savez_compressed(os.path.join(HERE, "dense_cases.npz"), **arrays)


def gen_rope(ref):
    """RoPE on one new token per sequence at scattered positions (rotary.py:29-109)."""
    arrays = {}
    for dt, (d, H) in C.ROPE_CASES.items():
        dtype = C.DTYPES[dt]
        x = C.rope_inputs(dt)
        inv = ref["build_inv_freq"](d, C.THETA, torch.device("cpu"))
        outs, coss, sins = [], [], []
        for i, p in enumerate(C.ROPE_POSITIONS):
            cos, sin = ref["build_rope_cache"](1, d, C.THETA, torch.device("cpu"), dtype, p, inv)
            o, _ = ref["apply_rotary"](x[i:i + 1], x[i:i + 1], cos, sin)
            outs.append(o)
            coss.append(cos)
            sins.append(sin)
        arrays[f"{dt}__sha"] = np.array(C.sha(x))
        arrays[f"{dt}__out"] = C.to_np(torch.cat(outs))
        arrays[f"{dt}__cos"] = C.to_np(torch.cat(coss))
        arrays[f"{dt}__sin"] = C.to_np(torch.cat(sins))
        arrays[f"{dt}__inv_freq"] = C.to_np(inv)
    np.savez_compressed(os.path.join(HERE, "rope_cases.npz"), **arrays)


def gen_tiny_model(ref):
    """Paged-cache decode parity of a tiny random Llama 3 (tests/test_llama3_shapes.py:152-198):
    weights, ids and the reference's full-forward logits for the decoded positions."""
    torch.manual_seed(126)
    cfg = ref["Llama3Config"](vocab_size=512, hidden_size=128, intermediate_size=256,
                              num_hidden_layers=2, num_attention_heads=8,
                              num_key_value_heads=4, max_position_embeddings=256)
    model = ref["Llama3ForCausalLM"](cfg)
    model.eval()
    ids = torch.randint(0, cfg.vocab_size, (1, 12))
    with torch.no_grad():
        full = model(input_ids=ids)["logits"]
        prefill = 8
        cache = ref["PagedKVCache"].create(cfg.num_hidden_layers, cfg.num_key_value_heads,
                                           cfg.head_dim, 32, 4, torch.device("cpu"), torch.float32)
        model(input_ids=ids[:, :prefill], past_key_values=cache, use_cache=True)
        steps = []
        for i in range(prefill, ids.shape[1]):
            steps.append(model(input_ids=ids[:, i:i + 1], past_key_values=cache,
                               use_cache=True)["logits"])
    step_logits = torch.cat(steps, dim=1)
    assert torch.allclose(step_logits, full[:, prefill:], atol=1e-5, rtol=1e-5)
    sd = {f"w__{k}": v.numpy() for k, v in model.state_dict().items()}
    np.savez_compressed(
        os.path.join(HERE, "tiny_llama_fp32.npz"), ids=ids.numpy(), prefill=prefill,
        full_logits=full.numpy(), step_logits=step_logits.numpy(),
        cfg=np.array([cfg.vocab_size, cfg.hidden_size, cfg.intermediate_size,
                      cfg.num_hidden_layers, cfg.num_attention_heads, cfg.num_key_value_heads]),
        **sd)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-src", default=os.environ.get("LLMCUDA_REF_SRC"),
                    help="the reference's src/ directory (or set LLMCUDA_REF_SRC)")
    args = ap.parse_args()
    if not args.ref_src:
        ap.error("pass --ref-src <llm-cuda>/src or set LLMCUDA_REF_SRC")
    sys.path.insert(0, args.ref_src)
    from llm_cuda.models.llama3 import attention as ra
    from llm_cuda.models.llama3 import kv_cache as rk
    from llm_cuda.models.llama3 import rotary as rr
    from llm_cuda.models.llama3.config import Llama3Config
    from llm_cuda.models.llama3.model import Llama3ForCausalLM

    ref = {
        "Llama3Attention": ra.Llama3Attention,
        "PagedKVLayerCache": rk.PagedKVLayerCache,
        "PagedKVCache": rk.PagedKVCache,
        "build_inv_freq": rr.build_inv_freq,
        "build_rope_cache": rr.build_rope_cache,
        "apply_rotary": rr.apply_rotary,
        "Llama3Config": Llama3Config,
        "Llama3ForCausalLM": Llama3ForCausalLM,
    }
    torch.set_num_threads(1)  # deterministic reductions for the fixtures
    gen_c1(ref)
    gen_step_cases(ref)
    gen_dense_cases(ref)
    gen_rope(ref)
    gen_tiny_model(ref)
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
