"""GPU parity of the CUDA decode path against the reference (golden fixtures) and the oracle.

Every case runs through the C ABI (``llm_cuda_b200._native`` -> libllmcuda_b200.so).
Tolerances are the north star's: fp32 1e-5 relative, bf16 2e-2 absolute (fp16:
the reference's own 1e-2).
"""

import math
import os

import numpy as np
import pytest
import torch

import cases as C
from helpers import TOL, assert_parity, fill_pages, oracle_decode, poison, to_f32_np
from llm_cuda_b200 import _native as N
from llm_cuda_b200.kernels.decode_attention import (
    can_use_triton_decode_attention,
    paged_decode,
    triton_decode_attention,
)
from llm_cuda_b200.models.llama3 import PagedKVLayerCache, RopeTable, make_block_table
from oracle import decode_oracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
DEV = torch.device("cuda", 0)


def _gold(name):
    return np.load(os.path.join(GOLD, name))


def _t(a, dt):
    return C.to_torch(a, dt).to(DEV)


# ---------------------------------------------------------------------------
# Config 1: fp32, 64-token prefill + 16 decode steps, permuted 8-page pool
# ---------------------------------------------------------------------------
def test_c1_full_path_matches_reference():
    g = _gold("c1_fp32.npz")
    q, k, v, perm = C.c1_inputs()
    q, k, v = q.to(DEV), k.to(DEV), v.to(DEV)
    bt = perm[:2].view(1, 2)
    cache = PagedKVLayerCache(2, 64, 80, 64, DEV, torch.float32, num_pages=8, block_table=bt)
    poison(cache)
    rope = RopeTable(80, 64, C.THETA, DEV, torch.float32)
    cache.append_rotary(q[:, :, :64], k[:, :, :64], v[:, :, :64], rope)
    outs, qrots = [], []
    for t in range(16):
        i = 64 + t
        q_rot = cache.append_rotary(q[:, :, i:i + 1], k[:, :, i:i + 1], v[:, :, i:i + 1], rope)
        outs.append(cache.decode(q_rot))
        qrots.append(q_rot)
    cache.check_status()
    assert cache.length == 80
    np.testing.assert_array_equal(to_f32_np(torch.stack(qrots)), g["q_rot"])
    np.testing.assert_allclose(to_f32_np(torch.stack(outs)), g["out"], **TOL["fp32"])
    kc, vc = cache.get_kv()
    np.testing.assert_array_equal(to_f32_np(kc), g["k_cache"])
    np.testing.assert_array_equal(to_f32_np(vc), g["v_cache"])


# ---------------------------------------------------------------------------
# Single decode steps on ragged batches vs the reference's outputs
# ---------------------------------------------------------------------------
def _step_case(name, partition_tokens=None, force_generic=False):
    dt, Hq, Hkv, d, lens, scale, seed = C.STEP_CASES[name]
    dtype = C.DTYPES[dt]
    seqs = C.step_inputs(name)
    P = 16
    B = len(lens)
    max_len = max(lens) + 16
    max_pages = math.ceil(max_len / P)
    gen = torch.Generator().manual_seed(seed)
    num_pages = B * max_pages + 5
    bt = make_block_table(B, max_pages, num_pages, max_pages, generator=gen)
    cache = PagedKVLayerCache(Hkv, d, max_len, P, DEV, dtype, batch_size=B, num_pages=num_pages,
                              block_table=bt)
    poison(cache)
    fill_pages(cache, [s[0] for s in seqs], [s[1] for s in seqs])
    rope = RopeTable(max_len, d, C.THETA, DEV, dtype)
    q = torch.stack([s[2] for s in seqs])[:, :, None].to(DEV)
    k = torch.stack([s[3] for s in seqs])[:, :, None].to(DEV)
    v = torch.stack([s[4] for s in seqs])[:, :, None].to(DEV)
    q_rot = cache.append_rotary(q, k, v, rope)
    out = paged_decode(q_rot, cache.key_pages, cache.value_pages, cache.block_table,
                       cache.seq_lens, host_lens=cache.host_lengths,
                       partition_tokens=partition_tokens, force_generic=force_generic,
                       status=cache.status)
    cache.check_status()
    assert cache.seq_lens.tolist() == lens
    return cache, q_rot, out


@pytest.mark.parametrize("variant", ["auto", "split64", "split128", "generic"])
@pytest.mark.parametrize("name", list(C.STEP_CASES))
def test_step_matches_reference(name, variant):
    dt = C.STEP_CASES[name][0]
    kw = {"auto": {}, "split64": {"partition_tokens": 64}, "split128": {"partition_tokens": 128},
          "generic": {"force_generic": True}}[variant]
    cache, q_rot, out = _step_case(name, **kw)
    g = _gold(f"step_{name}.npz")
    # RoPE: same rounding points as the reference's torch path -> bit-exact
    np.testing.assert_array_equal(C.to_np(q_rot[:, :, 0]), g["q_rot"])
    lens = C.STEP_CASES[name][4]
    for b, L in enumerate(lens):
        pos = L - 1
        page = int(cache.block_table[b, pos // 16])
        kstored = cache.key_pages[page, :, pos % 16]
        np.testing.assert_array_equal(C.to_np(kstored), g["k_rot"][b])
    ref = O.from_bits(g["out"], dt)
    assert_parity(out[:, :, 0], ref, C.DTYPES[dt], f"{name}/{variant}")


# ---------------------------------------------------------------------------
# Reference kernel test shapes through the dense entry point
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("name", list(C.DENSE_CASES))
def test_dense_entry_matches_reference(name):
    B, Hq, Hkv, L, d, dt = C.DENSE_CASES[name]
    q, k, v = (x.to(DEV) for x in C.dense_inputs(name))
    assert can_use_triton_decode_attention(q, k, v)
    out = triton_decode_attention(q, k, v)
    assert out.shape == q.shape and out.dtype == q.dtype
    ref = O.from_bits(_gold("dense_cases.npz")[f"{name}__out"], dt)
    assert_parity(out, ref, q.dtype, name)


def test_predicate_rejects_like_reference():
    q = torch.randn(1, 4, 1, 16, device=DEV, dtype=torch.float16)
    k = torch.randn(1, 2, 8, 16, device=DEV, dtype=torch.float16)
    assert can_use_triton_decode_attention(q, k, k)
    assert not can_use_triton_decode_attention(q.expand(1, 4, 3, 16), k, k)
    assert not can_use_triton_decode_attention(q, k[:, :, :0], k[:, :, :0])
    assert not can_use_triton_decode_attention(q.double(), k.double(), k.double())
    q5 = torch.randn(1, 5, 1, 16, device=DEV, dtype=torch.float16)
    k3 = torch.randn(1, 3, 8, 16, device=DEV, dtype=torch.float16)
    assert not can_use_triton_decode_attention(q5, k3, k3)
    assert not can_use_triton_decode_attention(
        torch.randn(1, 4, 1, 512, device=DEV, dtype=torch.float16),
        torch.randn(1, 2, 8, 512, device=DEV, dtype=torch.float16),
        torch.randn(1, 2, 8, 512, device=DEV, dtype=torch.float16))


# ---------------------------------------------------------------------------
# BASELINE configs at full size (oracle on every sequence + properties)
# ---------------------------------------------------------------------------
def _random_paged(B, Hq, Hkv, d, lens, P, dtype, seed, scale=1.0, pool_slack=7):
    gen = torch.Generator().manual_seed(seed)
    pages_per = [math.ceil(L / P) for L in lens]
    max_pages = max(pages_per)
    num_pages = sum(pages_per) + pool_slack
    bt = make_block_table(B, pages_per, num_pages, max_pages, generator=gen)
    cache = PagedKVLayerCache(Hkv, d, max_pages * P, P, DEV, dtype, batch_size=B,
                              num_pages=num_pages, block_table=bt)
    gd = torch.Generator(device=DEV).manual_seed(seed)
    cache.key_pages.normal_(generator=gd).mul_(scale)
    cache.value_pages.normal_(generator=gd).mul_(scale)
    cache.seq_lens.copy_(torch.tensor(lens, dtype=torch.int32))
    cache.host_lengths = list(lens)
    q = (torch.randn(B, Hq, d, device=DEV, generator=gd) * scale).to(dtype)
    return cache, q


def _logical(cache, b):
    L = cache.host_lengths[b]
    P = cache.page_size
    n = math.ceil(L / P)
    pages = cache.block_table[b, :n].long()
    k = cache.key_pages[pages].permute(1, 0, 2, 3).reshape(cache.num_kv_heads, n * P, -1)[:, :L]
    v = cache.value_pages[pages].permute(1, 0, 2, 3).reshape(cache.num_kv_heads, n * P, -1)[:, :L]
    return k.cpu(), v.cpu()


def _check_samples(cache, q, out, samples, what, chunk=16):
    """Oracle parity of the sequences ``samples``, ``chunk`` at a time (bounded host
    memory for the full-size configs)."""
    samples = list(samples)
    for i in range(0, len(samples), chunk):
        part = samples[i:i + chunk]
        ks, vs = zip(*[_logical(cache, b) for b in part])
        ref = oracle_decode(q[part].cpu(), ks, vs)
        assert_parity(out[part], ref, q.dtype, f"{what} sequences {part[0]}..{part[-1]}")


def test_config2_llama8b_full_size():
    """B64 Hq32 Hkv8 d128, L=4096, page 16, shuffled 16384-page pool."""
    cache, q = _random_paged(64, 32, 8, 128, [4096] * 64, 16, torch.bfloat16, 2002)
    out = cache.decode(q[:, :, None])[:, :, 0]
    cache.check_status()
    _check_samples(cache, q, out, range(64), "config2")          # every sequence
    # every sequence: the split-K/TMA kernel agrees with the SIMT kernel and with a
    # single-partition run (size-independent properties)
    gen = paged_decode(q, cache.key_pages, cache.value_pages, cache.block_table, cache.seq_lens,
                       force_generic=True, status=cache.status)
    one = paged_decode(q, cache.key_pages, cache.value_pages, cache.block_table, cache.seq_lens,
                       partition_tokens=4096, status=cache.status)
    cache.check_status()
    assert (out.float() - gen.float()).abs().max().item() < 2e-2
    assert (out.float() - one.float()).abs().max().item() < 2e-2
    # moving pages to other physical slots changes nothing (bit-exact)
    perm = torch.randperm(cache.num_pages, generator=torch.Generator().manual_seed(5)).to(DEV)
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(cache.num_pages, device=DEV)
    kp2 = torch.empty_like(cache.key_pages)
    vp2 = torch.empty_like(cache.value_pages)
    kp2[inv] = cache.key_pages
    vp2[inv] = cache.value_pages
    bt2 = inv[cache.block_table.long()].to(torch.int32)
    moved = paged_decode(q, kp2, vp2, bt2, cache.seq_lens, host_lens=cache.host_lengths,
                         status=cache.status)
    assert torch.equal(moved, out)


def test_config3_ragged_full_size():
    """B256, L ~ U[128, 32768] from the seed, page 16, shared pool in random order."""
    g = torch.Generator().manual_seed(1003)
    lens = torch.randint(128, 32769, (256,), generator=g).tolist()
    cache, q = _random_paged(256, 32, 8, 128, lens, 16, torch.bfloat16, 2003)
    out = cache.decode(q[:, :, None])[:, :, 0]
    cache.check_status()
    _check_samples(cache, q, out, range(256), "config3")         # every sequence
    gen = paged_decode(q, cache.key_pages, cache.value_pages, cache.block_table, cache.seq_lens,
                       force_generic=True, status=cache.status)
    assert (out.float() - gen.float()).abs().max().item() < 2e-2


def test_config4_long_context_split_k():
    """B4 Hq64 Hkv8 d128, L=131072, page 64, 4096-token partitions + LSE merge, x0.5."""
    cache, q = _random_paged(4, 64, 8, 128, [131072] * 4, 64, torch.bfloat16, 2004, scale=0.5)
    out = paged_decode(q, cache.key_pages, cache.value_pages, cache.block_table, cache.seq_lens,
                       partition_tokens=4096, status=cache.status)
    cache.check_status()
    _check_samples(cache, q, out, range(4), "config4", chunk=1)   # every sequence
    auto = cache.decode(q[:, :, None])[:, :, 0]
    assert (out.float() - auto.float()).abs().max().item() < 2e-2


# ---------------------------------------------------------------------------
# Edge cases and device-side error reporting
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("force_generic", [False, True])
def test_empty_and_short_contexts(force_generic):
    lens = [0, 1, 2, 15, 16, 17, 63, 64, 65, 257]
    cache, q = _random_paged(len(lens), 32, 8, 128, [max(L, 1) for L in lens], 16,
                             torch.bfloat16, 2005)
    cache.seq_lens.copy_(torch.tensor(lens, dtype=torch.int32))
    cache.host_lengths = list(lens)
    out = paged_decode(q, cache.key_pages, cache.value_pages, cache.block_table, cache.seq_lens,
                       partition_tokens=64, force_generic=force_generic, status=cache.status)
    cache.check_status()
    assert torch.count_nonzero(out[0]) == 0          # empty context -> zeros
    _check_samples(cache, q, out, list(range(1, len(lens))), "short")


# ---------------------------------------------------------------------------
# Balanced split (partition_tokens = 0): equal chunk ranges per CTA
# ---------------------------------------------------------------------------
BALANCED_CASES = {
    # name: (B, Hq, Hkv, d, lens, page, dtype)
    "fewer_chunks_than_ctas": (1, 8, 8, 128, [100], 16, torch.bfloat16),
    "two_head_groups": (3, 64, 4, 128, [5000, 0, 3000], 16, torch.bfloat16),
    "d64_page8_ragged": (5, 32, 8, 64, [1, 64, 65, 7000, 129], 8, torch.bfloat16),
    "d256_page32": (2, 16, 2, 256, [20000, 333], 32, torch.bfloat16),
    "page128_fp16": (7, 32, 8, 128, [128, 4096, 17, 9000, 1, 2048, 3333], 128, torch.float16),
    "one_row_many_ctas": (1, 4, 1, 128, [131072], 64, torch.bfloat16),
}


@pytest.mark.parametrize("name", list(BALANCED_CASES))
def test_balanced_split_matches_oracle(name):
    B, Hq, Hkv, d, lens, P, dtype = BALANCED_CASES[name]
    cache, q = _random_paged(B, Hq, Hkv, d, [max(L, 1) for L in lens], P, dtype, 2100)
    cache.seq_lens.copy_(torch.tensor(lens, dtype=torch.int32))
    cache.host_lengths = list(lens)
    lib = N.load()
    assert lib.llmc_decode_balanced_supported(q.data_ptr(), cache.key_pages.data_ptr(),
                                              cache.value_pages.data_ptr(),
                                              N.dtype_code(dtype), d, P, cache.max_pages, B)
    out = paged_decode(q, cache.key_pages, cache.value_pages, cache.block_table, cache.seq_lens,
                       partition_tokens=0, status=cache.status, workspace=cache.workspace)
    cache.check_status()
    # the in-kernel merge leaves its counters at zero, so a second call is identical
    rows = B * Hkv * ((Hq // Hkv + 7) // 8)
    words = ((rows + 1) + 31) // 32 * 32
    counters = cache.workspace.part_lse[:words].view(torch.int32)
    assert torch.count_nonzero(counters) == 0
    again = paged_decode(q, cache.key_pages, cache.value_pages, cache.block_table,
                         cache.seq_lens, partition_tokens=0, status=cache.status,
                         workspace=cache.workspace)
    assert torch.equal(again, out)
    for b, L in enumerate(lens):
        if L == 0:
            assert torch.count_nonzero(out[b]) == 0
    live = [b for b, L in enumerate(lens) if L > 0]
    _check_samples(cache, q, out, live, f"balanced/{name}")
    # the same rows through the SIMT kernel with uniform partitions
    gen = paged_decode(q, cache.key_pages, cache.value_pages, cache.block_table, cache.seq_lens,
                       partition_tokens=1024, force_generic=True, status=cache.status)
    assert (out.float() - gen.float()).abs().max().item() < 2e-2


def test_balanced_split_rejects_simt_only_shapes():
    """fp32 has no TMA kernel: the explicit balanced split is refused, not emulated."""
    cache, q = _random_paged(2, 8, 2, 128, [300, 40], 16, torch.float32, 2101)
    with pytest.raises(N.NativeLibraryError, match="balanced"):
        paged_decode(q, cache.key_pages, cache.value_pages, cache.block_table, cache.seq_lens,
                     partition_tokens=0, status=cache.status)
    # the default picks uniform partitions for this shape
    out = paged_decode(q, cache.key_pages, cache.value_pages, cache.block_table, cache.seq_lens,
                       host_lens=[300, 40], status=cache.status)
    cache.check_status()
    _check_samples(cache, q, out, [0, 1], "fp32 default")


def test_bad_page_is_reported_not_faulted():
    cache, q = _random_paged(2, 8, 2, 128, [100, 100], 16, torch.bfloat16, 2006)
    cache.block_table[1, 3] = cache.num_pages + 1000
    paged_decode(q, cache.key_pages, cache.value_pages, cache.block_table, cache.seq_lens,
                 status=cache.status)
    with pytest.raises(N.DeviceStatusError, match="page id"):
        cache.check_status()
    cache.check_status()  # cleared


def test_append_overflow_is_reported():
    cache = PagedKVLayerCache(2, 64, 32, 16, DEV, torch.bfloat16)
    cache.seq_lens.fill_(32)               # device says full, host mirror does not
    k = torch.zeros(1, 2, 1, 64, device=DEV, dtype=torch.bfloat16)
    cache.append(k, k)
    with pytest.raises(N.DeviceStatusError, match="capacity"):
        cache.check_status()
    with pytest.raises(ValueError):
        cache.append(torch.zeros(1, 2, 40, 64, device=DEV, dtype=torch.bfloat16),
                     torch.zeros(1, 2, 40, 64, device=DEV, dtype=torch.bfloat16))


def test_decode_step_graph_capture():
    """RoPE+append+decode+merge captured once and replayed: same result as eager."""
    B, Hq, Hkv, d, P = 8, 32, 8, 128, 16
    lens = [300 + 37 * i for i in range(B)]
    cache, _ = _random_paged(B, Hq, Hkv, d, [L + 8 for L in lens], P, torch.bfloat16, 2007)
    cache.seq_lens.copy_(torch.tensor(lens, dtype=torch.int32))
    cache.host_lengths = list(lens)
    rope = RopeTable(cache.max_seq_len, d, C.THETA, DEV, torch.bfloat16)
    gd = torch.Generator(device=DEV).manual_seed(7)
    q = torch.randn(B, Hq, 1, d, device=DEV, generator=gd).bfloat16()
    k = torch.randn(B, Hkv, 1, d, device=DEV, generator=gd).bfloat16()
    v = torch.randn(B, Hkv, 1, d, device=DEV, generator=gd).bfloat16()
    q_rot = torch.empty_like(q)
    out = torch.empty_like(q)
    kp0, vp0 = cache.key_pages.clone(), cache.value_pages.clone()
    # eager reference run
    cache.append_rotary(q, k, v, rope, q_out=q_rot)
    eager = cache.decode(q_rot, partition_tokens=128).clone()
    # reset and capture
    cache.key_pages.copy_(kp0)
    cache.value_pages.copy_(vp0)
    cache.seq_lens.copy_(torch.tensor(lens, dtype=torch.int32))
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            cache.append_rotary(q, k, v, rope, q_out=q_rot)
            cache.decode(q_rot, out=out.view(B, Hq, d), partition_tokens=128)
    torch.cuda.current_stream().wait_stream(s)
    cache.key_pages.copy_(kp0)
    cache.value_pages.copy_(vp0)
    cache.seq_lens.copy_(torch.tensor(lens, dtype=torch.int32))
    graph.replay()
    torch.cuda.synchronize()
    cache.check_status()
    assert torch.equal(out, eager)
    assert cache.seq_lens.tolist() == [L + 1 for L in lens]



# ---------------------------------------------------------------------------
# Fused RoPE + append + decode (llmc_rope_append_decode)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("T", [None, 64])
@pytest.mark.parametrize("name", list(C.STEP_CASES))
def test_fused_step_matches_reference(name, T):
    dt, Hq, Hkv, d, lens, scale, seed = C.STEP_CASES[name]
    dtype = C.DTYPES[dt]
    seqs = C.step_inputs(name)
    P, B = 16, len(lens)
    max_len = max(lens) + 16
    max_pages = math.ceil(max_len / P)
    gen = torch.Generator().manual_seed(seed)
    num_pages = B * max_pages + 5
    bt = make_block_table(B, max_pages, num_pages, max_pages, generator=gen)
    cache = PagedKVLayerCache(Hkv, d, max_len, P, DEV, dtype, batch_size=B, num_pages=num_pages,
                              block_table=bt)
    poison(cache)
    fill_pages(cache, [s[0] for s in seqs], [s[1] for s in seqs])
    rope = RopeTable(max_len, d, C.THETA, DEV, dtype)
    q = torch.stack([s[2] for s in seqs])[:, :, None].to(DEV)
    k = torch.stack([s[3] for s in seqs])[:, :, None].to(DEV)
    v = torch.stack([s[4] for s in seqs])[:, :, None].to(DEV)
    q_rot = torch.empty(B, Hq, d, device=DEV, dtype=dtype)
    out = cache.rope_append_decode(q, k, v, rope, q_out=q_rot, partition_tokens=T)
    cache.check_status()
    assert cache.seq_lens.tolist() == lens and cache.host_lengths == lens
    g = _gold(f"step_{name}.npz")
    np.testing.assert_array_equal(C.to_np(q_rot), g["q_rot"])
    for b, L in enumerate(lens):
        page = int(cache.block_table[b, (L - 1) // 16])
        np.testing.assert_array_equal(C.to_np(cache.key_pages[page, :, (L - 1) % 16]), g["k_rot"][b])
    assert_parity(out[:, :, 0], O.from_bits(g["out"], dt), dtype, f"fused/{name}")


def test_fused_step_equals_separate_kernels_config2():
    """Config 2 at full size: the fused step and append_rotary + decode give identical
    outputs, pages and lengths (the same rounding and the same reduction order)."""
    cache, _ = _random_paged(64, 32, 8, 128, [4096] * 64, 16, torch.bfloat16, 2010)
    lens0 = torch.full((64,), 4095, dtype=torch.int32, device=DEV)
    cache.seq_lens.copy_(lens0)
    cache.host_lengths = [4095] * 64
    rope = RopeTable(4096, 128, C.THETA, DEV, torch.bfloat16)
    gd = torch.Generator(device=DEV).manual_seed(3)
    q = torch.randn(64, 32, 1, 128, device=DEV, generator=gd).bfloat16()
    k = torch.randn(64, 8, 1, 128, device=DEV, generator=gd).bfloat16()
    v = torch.randn(64, 8, 1, 128, device=DEV, generator=gd).bfloat16()
    kp0, vp0 = cache.key_pages.clone(), cache.value_pages.clone()
    fused = cache.rope_append_decode(q, k, v, rope).clone()
    kp1, vp1, l1 = cache.key_pages.clone(), cache.value_pages.clone(), cache.seq_lens.clone()
    cache.key_pages.copy_(kp0)
    cache.value_pages.copy_(vp0)
    cache.seq_lens.copy_(lens0)
    cache.host_lengths = [4095] * 64
    sep = cache.decode(cache.append_rotary(q, k, v, rope))
    cache.check_status()
    assert torch.equal(cache.seq_lens, l1) and l1.tolist() == [4096] * 64
    assert torch.equal(cache.key_pages, kp1) and torch.equal(cache.value_pages, vp1)
    assert torch.equal(fused, sep)


def test_fused_step_graph_replay():
    B, Hq, Hkv, d, P = 8, 32, 8, 128, 16
    lens = [300 + 37 * i for i in range(B)]
    cache, _ = _random_paged(B, Hq, Hkv, d, [L + 8 for L in lens], P, torch.bfloat16, 2011)
    rope = RopeTable(cache.max_seq_len, d, C.THETA, DEV, torch.bfloat16)
    gd = torch.Generator(device=DEV).manual_seed(8)
    q = torch.randn(B, Hq, 1, d, device=DEV, generator=gd).bfloat16()
    k = torch.randn(B, Hkv, 1, d, device=DEV, generator=gd).bfloat16()
    v = torch.randn(B, Hkv, 1, d, device=DEV, generator=gd).bfloat16()
    out = torch.empty(B, Hq, d, device=DEV, dtype=torch.bfloat16)
    kp0, vp0 = cache.key_pages.clone(), cache.value_pages.clone()

    def reset():
        cache.key_pages.copy_(kp0)
        cache.value_pages.copy_(vp0)
        cache.seq_lens.copy_(torch.tensor(lens, dtype=torch.int32))
        cache.host_lengths = list(lens)

    reset()
    eager = cache.rope_append_decode(q, k, v, rope, partition_tokens=128).clone()
    reset()
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            cache.rope_append_decode(q, k, v, rope, out=out, partition_tokens=128)
    torch.cuda.current_stream().wait_stream(s)
    reset()
    graph.replay()
    torch.cuda.synchronize()
    cache.check_status()
    assert torch.equal(out.view_as(eager), eager)
    assert cache.seq_lens.tolist() == [L + 1 for L in lens]


def test_graphed_decode_step_matches_eager_two_steps():
    from llm_cuda_b200.models.llama3.kv_cache import GraphedDecodeStep

    B, Hq, Hkv, d, P = 6, 32, 8, 128, 16
    lens = [100 + 50 * i for i in range(B)]
    cache, _ = _random_paged(B, Hq, Hkv, d, [L + 8 for L in lens], P, torch.bfloat16, 2012)
    rope = RopeTable(cache.max_seq_len, d, C.THETA, DEV, torch.bfloat16)
    gd = torch.Generator(device=DEV).manual_seed(9)
    qs = [torch.randn(B, Hq, 1, d, device=DEV, generator=gd).bfloat16() for _ in range(2)]
    ks = [torch.randn(B, Hkv, 1, d, device=DEV, generator=gd).bfloat16() for _ in range(2)]
    vs = [torch.randn(B, Hkv, 1, d, device=DEV, generator=gd).bfloat16() for _ in range(2)]
    kp0, vp0 = cache.key_pages.clone(), cache.value_pages.clone()

    def reset():
        cache.key_pages.copy_(kp0)
        cache.value_pages.copy_(vp0)
        cache.seq_lens.copy_(torch.tensor(lens, dtype=torch.int32))
        cache.host_lengths = list(lens)

    reset()
    eager = [cache.rope_append_decode(qs[i], ks[i], vs[i], rope, partition_tokens=128).clone()
             for i in range(2)]
    reset()
    qb, kb, vb = torch.empty_like(qs[0]), torch.empty_like(ks[0]), torch.empty_like(vs[0])
    step = GraphedDecodeStep(cache, rope, qb, kb, vb, partition_tokens=128)
    for i in range(2):
        qb.copy_(qs[i])
        kb.copy_(ks[i])
        vb.copy_(vs[i])
        out = step.replay()
        torch.cuda.synchronize()
        assert torch.equal(out.view_as(eager[i]), eager[i])
    cache.check_status()
    assert cache.seq_lens.tolist() == [L + 2 for L in lens] and cache.host_lengths == [L + 2 for L in lens]


def test_fused_balanced_steps_match_uniform_partitions():
    """Six fused steps with the balanced split (in-kernel merge, lengths published by
    the decode launch) against the same steps with uniform 128-token partitions;
    contexts cross 64-token chunk edges and include an empty one."""
    B, Hq, Hkv, d, P = 6, 32, 8, 128, 16
    lens = [0, 62, 63, 64, 1000, 4093]
    cache, _ = _random_paged(B, Hq, Hkv, d, [L + 8 for L in lens], P, torch.bfloat16, 2013)
    rope = RopeTable(cache.max_seq_len, d, C.THETA, DEV, torch.bfloat16)
    gd = torch.Generator(device=DEV).manual_seed(13)
    kp0, vp0 = cache.key_pages.clone(), cache.value_pages.clone()
    steps = [tuple(torch.randn(B, h, 1, d, device=DEV, generator=gd).bfloat16()
                   for h in (Hq, Hkv, Hkv)) for _ in range(6)]

    def run(T):
        cache.key_pages.copy_(kp0)
        cache.value_pages.copy_(vp0)
        cache.seq_lens.copy_(torch.tensor(lens, dtype=torch.int32))
        cache.host_lengths = list(lens)
        outs = [cache.rope_append_decode(q, k, v, rope, partition_tokens=T).clone()
                for q, k, v in steps]
        cache.check_status()
        assert cache.seq_lens.tolist() == [L + 6 for L in lens]
        return torch.stack(outs)

    bal = run(0)
    uni = run(128)
    assert (bal.float() - uni.float()).abs().max().item() < 2e-2
    assert torch.isfinite(bal.float()).all()
