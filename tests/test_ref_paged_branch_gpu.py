"""The paged decode branch inside the reference's own model.

``Llama3Attention.forward`` of the unmodified reference (``attention.py:91-150`` of
llm-cuda) gets the decode branch this package documents for it: for a paged cache and
one new token, the projections are followed by ONE RoPE + page-append launch
(``append_rotary``) and the paged flash-decode (``decode``), with no
``build_rope_cache``, no ``get_kv`` gather and no dense attention; every other call goes
to the reference's own forward.  The reference's ``Llama3ForCausalLM`` then decodes the
tiny fixture model token by token from position 0 (every forward is a decode step), and
its logits must equal the reference CPU model's at 1e-5 (fp32), the reference's own
decode-parity bar (``tests/test_llama3_shapes.py:152-198``).
"""

import numpy as np
import pytest
import torch

from test_dropin_reference_gpu import DEV, ref_model  # noqa: F401  (fixture)

pytestmark = pytest.mark.gpu


def test_reference_model_with_paged_decode_branch(ref_model, monkeypatch):  # noqa: F811
    model, g, _ = ref_model
    import llm_cuda.models.llama3.attention as ref_attention

    from llm_cuda_b200.models.llama3 import RopeTable
    from llm_cuda_b200.models.llama3.kv_cache import PagedKVCache, PagedKVLayerCache

    cfg = model.config
    rope = RopeTable(64, cfg.head_dim, cfg.rope_theta, DEV, torch.float32)
    orig = ref_attention.Llama3Attention.forward
    taken = {"n": 0}

    def forward(self, x, attention_mask=None, past_key_value=None, use_cache=False):
        bsz, seq_len, _ = x.shape
        if isinstance(past_key_value, PagedKVLayerCache) and seq_len == 1 and use_cache:
            q = self._shape(self.q_proj(x), self.num_heads)
            k = self._shape(self.k_proj(x), self.num_kv_heads)
            v = self._shape(self.v_proj(x), self.num_kv_heads)
            q = past_key_value.append_rotary(q, k, v, rope)    # RoPE(q, k) + page append
            out = past_key_value.decode(q)                     # paged GQA flash-decode
            out = out.transpose(1, 2).contiguous().view(bsz, 1, self.num_heads * self.head_dim)
            taken["n"] += 1
            return self.o_proj(out), past_key_value
        return orig(self, x, attention_mask, past_key_value, use_cache)

    monkeypatch.setattr(ref_attention.Llama3Attention, "forward", forward)
    ids = torch.from_numpy(g["ids"]).to(DEV)
    cache = PagedKVCache.create(num_layers=cfg.num_hidden_layers,
                                num_kv_heads=cfg.num_key_value_heads, head_dim=cfg.head_dim,
                                max_seq_len=32, page_size=4, device=DEV, dtype=torch.float32)
    steps = []
    with torch.no_grad():
        for t in range(ids.shape[1]):
            out = model(input_ids=ids[:, t:t + 1], past_key_values=cache, use_cache=True)
            steps.append(out["logits"][:, -1])
    cache.check_status()
    assert taken["n"] == ids.shape[1] * cfg.num_hidden_layers
    assert cache.get_layer(0).length == ids.shape[1]
    got = torch.stack(steps, dim=1).cpu().numpy()
    np.testing.assert_allclose(got, g["full_logits"], rtol=1e-5, atol=1e-5)
