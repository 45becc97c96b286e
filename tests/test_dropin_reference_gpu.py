"""Drop-in test: the reference's own Llama 3 decode loop with this package swapped in.

The unmodified reference model (``llm_cuda.models.llama3``, ``model.py:178-218`` and
``attention.py:91-150`` of llm-cuda) runs on the GPU with

* ``can_use_triton_decode_attention`` / ``triton_decode_attention``, the names
  ``attention.py:5-8`` imports, bound to this package's CUDA implementation, and
* ``PagedKVLayerCache`` / ``PagedKVCache``, the names ``attention.py:12`` and
  ``model.py:8`` import and ``isinstance``-check (``attention.py:105,121,130``,
  ``model.py:67,93,97``), bound to this package's paged cache,

exactly as a user of the reference would switch (the module attributes are
replaced; no reference file is edited).  The reference's other GPU kernels (Triton
RMSNorm, SwiGLU and RoPE, and its JIT CUDA extension) are put on their own torch
fallbacks, the branches the reference takes on a machine without Triton or the
extension, so every op outside the swapped path has the arithmetic of the
reference's CPU run that produced the fixture.  The logits are then held to the
reference's own decode-parity bar (``tests/test_llama3_shapes.py:152-198``:
1e-5 absolute and relative, fp32).
"""

import os

import numpy as np
import pytest
import torch

from refsrc import import_reference

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture
def ref_model(monkeypatch):
    llm_cuda = import_reference()
    if llm_cuda is None:
        pytest.skip("reference not installed in baseline/_ref (and LLMCUDA_REF_SRC unset)")
    import llm_cuda.kernels.cuda.extension as ref_ext
    import llm_cuda.kernels.triton.rope as ref_rope
    import llm_cuda.kernels.triton.swiglu as ref_swiglu
    import llm_cuda.models.llama3.attention as ref_attention
    import llm_cuda.models.llama3.model as ref_model_mod
    from llm_cuda.models.llama3.config import Llama3Config
    from llm_cuda.models.llama3.norm import RMSNorm

    from llm_cuda_b200.kernels import decode_attention as ours
    from llm_cuda_b200.models.llama3 import kv_cache as our_cache

    # the swap a user makes: decode attention + paged cache, rebound in the reference's modules
    monkeypatch.setattr(ref_attention, "can_use_triton_decode_attention",
                        ours.can_use_triton_decode_attention)
    monkeypatch.setattr(ref_attention, "triton_decode_attention", ours.triton_decode_attention)
    monkeypatch.setattr(ref_attention, "PagedKVLayerCache", our_cache.PagedKVLayerCache)
    monkeypatch.setattr(ref_model_mod, "PagedKVCache", our_cache.PagedKVCache)
    monkeypatch.setattr(ref_model_mod, "PagedKVLayerCache", our_cache.PagedKVLayerCache)
    # the reference's other kernels on their torch fallbacks (no Triton, no extension)
    import llm_cuda.kernels.cuda.attention as ref_cuda_attn
    import llm_cuda.kernels.cuda.rmsnorm as ref_cuda_norm
    import llm_cuda.kernels.cuda.swiglu as ref_cuda_swiglu

    for mod in (ref_ext, ref_cuda_attn, ref_cuda_norm, ref_cuda_swiglu):
        if hasattr(mod, "load_cuda_extension"):
            monkeypatch.setattr(mod, "load_cuda_extension", lambda verbose=False: None)
    monkeypatch.setattr(ref_swiglu, "triton", None)
    monkeypatch.setattr(ref_rope, "triton", None)

    g = np.load(os.path.join(GOLD, "tiny_llama_fp32.npz"))
    V, H, I, Lyr, Hq, Hkv = (int(x) for x in g["cfg"])
    cfg = Llama3Config(vocab_size=V, hidden_size=H, intermediate_size=I, num_hidden_layers=Lyr,
                       num_attention_heads=Hq, num_key_value_heads=Hkv,
                       max_position_embeddings=256)
    model = ref_model_mod.Llama3ForCausalLM(cfg)
    model.load_state_dict({k[3:]: torch.from_numpy(g[k]) for k in g.files if k.startswith("w__")})
    for m in model.modules():
        if isinstance(m, RMSNorm):
            m.use_triton = False
            m.use_cuda_extension = False
    model = model.to(DEV).eval()
    return model, g, ref_model_mod


def test_reference_decode_loop_with_paged_cache_swapped_in(ref_model):
    """The reference's paged decode parity flow, token by token from position 0 so that
    every step takes the decode branch (q_len == 1): each step's logits must equal the
    reference CPU model's full-sequence logits at that position."""
    model, g, ref_model_mod = ref_model
    from llm_cuda_b200.models.llama3.kv_cache import PagedKVCache, PagedKVLayerCache

    cfg = model.config
    ids = torch.from_numpy(g["ids"]).to(DEV)
    cache = ref_model_mod.PagedKVCache.create(
        num_layers=cfg.num_hidden_layers, num_kv_heads=cfg.num_key_value_heads,
        head_dim=cfg.head_dim, max_seq_len=32, page_size=4, device=DEV,
        dtype=model.model.embed_tokens.weight.dtype)
    assert isinstance(cache, PagedKVCache)
    assert isinstance(cache.get_layer(0), PagedKVLayerCache)
    calls = {"n": 0}
    import llm_cuda.models.llama3.attention as ref_attention

    real = ref_attention.triton_decode_attention

    def counted(q, k, v):
        calls["n"] += 1
        return real(q, k, v)

    ref_attention.triton_decode_attention = counted
    try:
        steps = []
        with torch.no_grad():
            for t in range(ids.shape[1]):
                out = model(input_ids=ids[:, t:t + 1], past_key_values=cache, use_cache=True)
                assert out["past_key_values"] is cache
                steps.append(out["logits"][:, -1])
    finally:
        ref_attention.triton_decode_attention = real
    cache.check_status()
    assert calls["n"] == ids.shape[1] * cfg.num_hidden_layers   # every layer, every step
    assert cache.get_layer(0).length == ids.shape[1]             # B = 1 ``.length``
    got = torch.stack(steps, dim=1).cpu().numpy()
    np.testing.assert_allclose(got, g["full_logits"], rtol=1e-5, atol=1e-5)
    prefill = int(g["prefill"])
    np.testing.assert_allclose(got[:, prefill:], g["step_logits"], rtol=1e-5, atol=1e-5)


def test_reference_generate_with_paged_cache_swapped_in(ref_model):
    """``Llama3ForCausalLM.generate(use_paged_kv=True)`` (model.py:178-218) builds the cache
    through the swapped ``PagedKVCache.create``; with a one-token prompt every forward is
    a decode step.  Greedy tokens must match the reference CPU logits' argmax."""
    model, g, _ = ref_model
    ids = torch.from_numpy(g["ids"]).to(DEV)
    out = model.generate(ids[:, :1], max_new_tokens=4, use_paged_kv=True, page_size=4)
    # the first generated token is the argmax of the reference logits at position 0
    assert int(out[0, 1]) == int(np.argmax(g["full_logits"][0, 0]))
    assert out.shape == (1, 5)
