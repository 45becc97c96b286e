"""GPU parity of the config-5 decode model (the caller of the decode path)."""

import os

import numpy as np
import pytest
import torch

from llm_cuda_b200.models.llama3.decode_model import DecodeConfig, DecodeGraph, Llama3DecodeModel
from llm_cuda_b200.models.llama3.rotary import build_rope_cache

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def test_tiny_llama_paged_decode_matches_reference():
    """Reference's own paged-decode parity test (tests/test_llama3_shapes.py:152-198):
    same weights and ids; the reference's logits come from its CPU model."""
    g = np.load(os.path.join(GOLD, "tiny_llama_fp32.npz"))
    V, H, I, Lyr, Hq, Hkv = (int(x) for x in g["cfg"])
    cfg = DecodeConfig(vocab_size=V, hidden_size=H, intermediate_size=I, num_hidden_layers=Lyr,
                       num_attention_heads=Hq, num_key_value_heads=Hkv)
    sd = {k[3:]: torch.from_numpy(g[k]) for k in g.files if k.startswith("w__")}
    m = Llama3DecodeModel.from_reference_state_dict(cfg, sd, DEV, torch.float32, max_positions=64)
    ids = torch.from_numpy(g["ids"]).to(DEV)
    prefill = int(g["prefill"])
    cache = m.make_cache(1, 32, page_size=4, shuffle_seed=3)
    last = m.prefill(ids[:, :prefill], cache)
    np.testing.assert_allclose(last.cpu().numpy(), g["full_logits"][:, prefill - 1], rtol=1e-5,
                               atol=1e-5)
    steps = [m.decode_step(ids[:, i], cache) for i in range(prefill, ids.shape[1])]
    cache.check_status()
    got = torch.stack(steps, dim=1).cpu().numpy()
    np.testing.assert_allclose(got, g["step_logits"], rtol=1e-5, atol=1e-5)


def _reference_attn_core(model):
    """The reference's decode branch on the GPU in the model dtype: torch RoPE
    (rotary.py:104-109), plain append, get_kv gather, _repeat_kv + _torch_attention
    (attention.py:56-89)."""

    def core(li, q, k, v, lc):
        pos = lc.length
        d = q.shape[-1]
        cos, sin = build_rope_cache(1, d, model.cfg.rope_theta, torch.device("cpu"), q.dtype, pos)
        cos, sin = cos.to(q.device)[None, None], sin.to(q.device)[None, None]

        def rot(x):
            h = x.shape[-1] // 2
            return (x * cos) + (torch.cat((-x[..., h:], x[..., :h]), -1) * sin)

        q, k = rot(q), rot(k)
        lc.append(k, v)
        kc, vc = lc.get_kv()
        rep = q.shape[1] // kc.shape[1]
        kc = kc.repeat_interleave(rep, dim=1)
        vc = vc.repeat_interleave(rep, dim=1)
        s = torch.matmul(q, kc.transpose(-2, -1)) / (d ** 0.5)
        return torch.matmul(torch.softmax(s, dim=-1), vc)

    return core


def test_llama8b_shape_step_matches_reference_attention():
    """Full Llama-3-8B layer shapes (2 layers), bf16, B=8: the fused CUDA attention path
    vs the reference's torch decode branch on identical weights and caches.  Layer 0
    sees identical inputs in both runs, so its attention output is held to the 2e-2
    bf16 bar; the logits after both layers are compared loosely (bf16 differences in
    layer 0 propagate) and by greedy agreement."""
    cfg = DecodeConfig(num_hidden_layers=2)
    m = Llama3DecodeModel.random_init(cfg, DEV, torch.bfloat16, seed=5, max_positions=512)
    B, S = 8, 200
    ids = torch.randint(0, cfg.vocab_size, (B, S), generator=torch.Generator().manual_seed(1)).to(DEV)
    cache = m.make_cache(B, 256, page_size=16, shuffle_seed=1)
    m.prefill(ids, cache)
    kp = [(lc.key_pages.clone(), lc.value_pages.clone(), lc.seq_lens.clone())
          for lc in cache.layer_caches]
    nxt = ids[:, -1]
    seen = {}

    def ours(li, q, k, v, lc):
        out = lc.decode(lc.append_rotary(q, k, v, m.rope))
        seen.setdefault(("ours", li), out.clone())
        return out

    ref_core = _reference_attn_core(m)

    def ref(li, q, k, v, lc):
        out = ref_core(li, q, k, v, lc)
        seen.setdefault(("ref", li), out.clone())
        return out

    m.attn_core = ours
    a = m.decode_step(nxt, cache).float()
    for lc, (k0, v0, l0) in zip(cache.layer_caches, kp):
        lc.key_pages.copy_(k0)
        lc.value_pages.copy_(v0)
        lc.seq_lens.copy_(l0)
        lc.host_lengths = [S] * B
    m.attn_core = ref
    b = m.decode_step(nxt, cache).float()
    m.attn_core = None
    cache.check_status()
    o_ref = seen[("ref", 0)].float()
    att = (seen[("ours", 0)].float() - o_ref).abs().max().item()
    print(f"\nlayer-0 attention max|ours - ref| = {att:.3e} (max|ref| {o_ref.abs().max().item():.2f})")
    assert att <= 2e-2, att
    scale = b.abs().max().item()
    assert (a - b).abs().max().item() <= 0.05 * scale
    assert (a.argmax(-1) == b.argmax(-1)).float().mean().item() >= 0.75


def test_decode_graph_replay_matches_eager():
    cfg = DecodeConfig(vocab_size=1000, hidden_size=512, intermediate_size=1024,
                       num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2)
    m = Llama3DecodeModel.random_init(cfg, DEV, torch.bfloat16, seed=9, max_positions=256)
    B, S, steps = 4, 40, 5
    ids = torch.randint(0, cfg.vocab_size, (B, S), generator=torch.Generator().manual_seed(2)).to(DEV)

    def run(graph: bool):
        cache = m.make_cache(B, 64, page_size=16, shuffle_seed=4)
        logits = m.prefill(ids, cache)
        nxt = logits.argmax(-1)
        out = []
        if graph:
            gr = DecodeGraph(m, cache, nxt, partition_tokens=64)
            for _ in range(steps):
                gr.replay()
                out.append(gr.next_ids.clone())
        else:
            for _ in range(steps):
                nxt = m.decode_step(nxt, cache, partition_tokens=64).argmax(-1)
                out.append(nxt.clone())
        torch.cuda.synchronize()
        cache.check_status()
        assert cache.get_layer(0).host_lengths == [S + steps] * B
        assert cache.get_layer(1).seq_lens.tolist() == [S + steps] * B
        return torch.stack(out)

    assert torch.equal(run(True), run(False))


@pytest.mark.parametrize("hidden", [4096, 8192 + 8, 100])   # 16-byte vectors x1 / x4; scalar
@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 2e-2)])
def test_add_rmsnorm_and_swiglu_match_torch_fp32(dtype, tol, hidden):
    from llm_cuda_b200.kernels.step_ops import add_rmsnorm, swiglu

    g = torch.Generator(device=DEV).manual_seed(3)
    x = torch.randn(64, 1, hidden, device=DEV, generator=g).to(dtype)
    dl = torch.randn(64, 1, hidden, device=DEV, generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(hidden, device=DEV, generator=g)).to(dtype)
    xs = (x.float() + dl.float()).to(dtype).float()          # residual stream in the dtype
    ref = xs * torch.rsqrt(xs.pow(2).mean(-1, keepdim=True) + 1e-5) * w.float()
    h = add_rmsnorm(x, w, 1e-5, delta=dl)
    torch.testing.assert_close(x.float(), xs)
    torch.testing.assert_close(h.float(), ref, rtol=tol, atol=tol)
    inter = hidden * 7 // 16                 # 1792: 16-byte vectors; 3587, 43: scalar path
    gu = torch.randn(64, 1, 2 * inter, device=DEV, generator=g).to(dtype)
    gg, uu = gu.float().split(inter, -1)
    torch.testing.assert_close(swiglu(gu).float(), gg * torch.sigmoid(gg) * uu, rtol=tol, atol=tol)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("rows,n", [(64, 128256), (3, 1000), (1, 7)])
def test_argmax_rows_matches_torch(dtype, rows, n):
    from llm_cuda_b200.kernels.step_ops import argmax_rows

    g = torch.Generator(device=DEV).manual_seed(rows + n)
    x = torch.randn(rows, n, device=DEV, generator=g).to(dtype)
    x[0, n // 2] = x[0, n // 3] = 100.0          # a tie: the first index wins
    for _ in range(2):                             # the workspace returns to zero
        got = argmax_rows(x)
        torch.testing.assert_close(got, torch.argmax(x, dim=-1))
    assert int(got[0]) == n // 3


def test_fused_step_reads_strided_qkv_views():
    """q/k/v as views into one fused QKV projection output (decode_step's layout) give
    the same step, bit for bit, as contiguous copies."""
    from llm_cuda_b200.models.llama3 import PagedKVLayerCache, RopeTable, make_block_table

    B, Hq, Hkv, d, P, L = 8, 32, 8, 128, 16, 777
    mp = (L + 64) // P
    gen = torch.Generator().manual_seed(5)
    bt = make_block_table(B, mp, B * mp + 3, mp, generator=gen)
    out = []
    qkv = torch.randn(B, 1, (Hq + 2 * Hkv) * d, device=DEV,
                      generator=torch.Generator(device=DEV).manual_seed(6)).bfloat16()
    q, k, v = qkv.split([Hq * d, Hkv * d, Hkv * d], dim=-1)
    views = [t.view(B, 1, h, d).transpose(1, 2) for t, h in ((q, Hq), (k, Hkv), (v, Hkv))]
    for strided in (True, False):
        c = PagedKVLayerCache(Hkv, d, mp * P, P, DEV, torch.bfloat16, batch_size=B,
                              num_pages=B * mp + 3, block_table=bt)
        gd = torch.Generator(device=DEV).manual_seed(7)
        c.key_pages.normal_(generator=gd)
        c.value_pages.normal_(generator=gd)
        c.seq_lens.fill_(L)
        c.host_lengths = [L] * B
        rope = RopeTable(mp * P, d, 500000.0, DEV, torch.bfloat16)
        qq, kk, vv = views if strided else [t.contiguous() for t in views]
        out.append((c.rope_append_decode(qq, kk, vv, rope).clone(), c.key_pages.clone()))
        c.check_status()
    assert torch.equal(out[0][0], out[1][0])
    assert torch.equal(out[0][1], out[1][1])
