"""The no-allocation decode entry point, for callers that cannot allocate device memory.

Some hosts of this library own all GPU memory themselves and hand a plugin only its
input and output buffers, so the plugin cannot call cudaMalloc or receive a split-K
workspace.  ``llmc_paged_decode_noalloc`` serves them with a scratch array built into
the library.  This test calls it through the C ABI twice in a row and checks each
result against the regular ``llmc_paged_decode`` + ``llmc_lse_merge`` path, within the
bf16 parity tolerance used by the other GPU tests (2e-2 absolute).  It sits in its
own file, collected last, and passes alone or after the rest of the suite.
"""

import math

import numpy as np
import pytest
import torch

from llm_cuda_b200 import _native as N
from llm_cuda_b200.kernels.decode_attention import paged_decode
from llm_cuda_b200.models.llama3 import make_block_table

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _case(seed, B=16, Hq=32, Hkv=8, d=128, P=16, max_len=1200, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(1, max_len + 1, (B,), generator=g).tolist()
    lens[0] = max_len                               # at least one multi-partition sequence
    max_pages = math.ceil(max_len / P)
    num_pages = B * max_pages + 3
    bt = make_block_table(B, max_pages, num_pages, max_pages, generator=g).to(DEV)
    gd = torch.Generator(device=DEV).manual_seed(seed)
    kp = torch.randn(num_pages, Hkv, P, d, device=DEV, generator=gd).to(dtype)
    vp = torch.randn(num_pages, Hkv, P, d, device=DEV, generator=gd).to(dtype)
    q = torch.randn(B, Hq, d, device=DEV, generator=gd).to(dtype)
    seq = torch.tensor(lens, dtype=torch.int32, device=DEV)
    return q, kp, vp, bt, seq, max_pages, num_pages


def _noalloc(q, kp, vp, bt, seq, max_pages, num_pages, T, out, status):
    lib = N.load()
    B, Hq, d = q.shape
    _, Hkv, P, _ = kp.shape
    return lib.llmc_paged_decode_noalloc(
        q.data_ptr(), kp.data_ptr(), vp.data_ptr(), bt.data_ptr(), seq.data_ptr(),
        out.data_ptr(), status.data_ptr(), B, Hq, Hkv, d, P, max_pages, num_pages, T,
        1.0 / math.sqrt(d), N.dtype_code(q.dtype), N.stream_handle(DEV))


def _oracle(q, kp, vp, bt, seq):
    """The CPU oracle (the reference's _repeat_kv + _torch_attention restated) on the
    logical K/V that the block table names."""
    from oracle import decode_oracle as O

    dt = {torch.bfloat16: "bf16", torch.float16: "fp16", torch.float32: "fp32"}[q.dtype]
    qn, kn, vn = (t.float().cpu().numpy() for t in (q, kp, vp))
    btn, lens = bt.cpu().numpy(), seq.tolist()
    return np.stack([O.decode_attention(qn[b], O.gather_logical(kn, btn[b], L),
                                        O.gather_logical(vn, btn[b], L), dt)
                     for b, L in enumerate(lens)])


def test_noalloc_matches_regular_entry_twice():
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    for call, seed in enumerate((11, 12)):           # two calls in a row, different inputs
        q, kp, vp, bt, seq, mp, npg = _case(seed)
        T = 256                                      # several partitions -> scratch is used
        ref = paged_decode(q, kp, vp, bt, seq, partition_tokens=T, status=status)
        out = torch.full_like(q, float("nan"))
        rc = _noalloc(q, kp, vp, bt, seq, mp, npg, T, out, status)
        assert rc == 0, N.load().llmc_last_error_string()
        torch.cuda.synchronize()
        N.raise_on_status(status)
        assert torch.isfinite(out.float()).all(), f"call {call}"
        err = (out.float() - ref.float()).abs().max().item()
        assert err <= 2e-2, f"call {call}: max abs diff {err}"


def test_noalloc_rejects_oversized_partials():
    lib = N.load()
    cap = lib.llmc_paged_decode_noalloc_capacity_bytes()
    assert cap == 8 << 20
    q, kp, vp, bt, seq, mp, npg = _case(13, B=4)
    out = torch.empty_like(q)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    # pretend a 4096-page table: 4 x 32 heads x 1024 partitions x 129 floats > 8 MiB
    rc = _noalloc(q, kp, vp, bt, seq, 4096, npg, 64, out, status)
    assert rc == -1
    assert b"scratch" in lib.llmc_last_error_string()


def test_noalloc_multi_partition_matches_oracle():
    """Several partitions per sequence land in the built-in scratch; the merged result is
    held to the CPU oracle at the bf16 bar (2e-2 absolute)."""
    q, kp, vp, bt, seq, mp, npg = _case(21, B=6, max_len=1000)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = torch.full_like(q, float("nan"))
    rc = _noalloc(q, kp, vp, bt, seq, mp, npg, 128, out, status)   # up to 8 partitions
    assert rc == 0, N.load().llmc_last_error_string()
    torch.cuda.synchronize()
    N.raise_on_status(status)
    np.testing.assert_allclose(out.float().cpu().numpy(), _oracle(q, kp, vp, bt, seq),
                               rtol=0.0, atol=2e-2)


@pytest.mark.parametrize("d", [64, 48])
def test_noalloc_fp32_generic_kernel_matches_regular_entry(d):
    """fp32 (and d=48) run the SIMT kernel through the scratch: same bits as the regular
    entry point, and within the fp32 bar (1e-5 relative) of the oracle."""
    q, kp, vp, bt, seq, mp, npg = _case(31, B=5, Hq=8, Hkv=2, d=d, max_len=700,
                                        dtype=torch.float32)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    for _ in range(2):
        ref = paged_decode(q, kp, vp, bt, seq, partition_tokens=192, status=status)
        out = torch.full_like(q, float("nan"))
        rc = _noalloc(q, kp, vp, bt, seq, mp, npg, 192, out, status)
        assert rc == 0, N.load().llmc_last_error_string()
        torch.cuda.synchronize()
        N.raise_on_status(status)
        assert torch.equal(out, ref)
    np.testing.assert_allclose(out.cpu().numpy(), _oracle(q, kp, vp, bt, seq),
                               rtol=1e-5, atol=1e-6)


def test_noalloc_single_partition_skips_merge():
    """partition_tokens covering the whole table: one partition, the decode kernel writes
    out directly and the merge leaves it alone."""
    q, kp, vp, bt, seq, mp, npg = _case(41, B=8, max_len=500)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    T = 64 * math.ceil(mp * 16 / 64)
    ref = paged_decode(q, kp, vp, bt, seq, partition_tokens=T, status=status)
    out = torch.full_like(q, float("nan"))
    rc = _noalloc(q, kp, vp, bt, seq, mp, npg, T, out, status)
    assert rc == 0, N.load().llmc_last_error_string()
    torch.cuda.synchronize()
    N.raise_on_status(status)
    assert (out.float() - ref.float()).abs().max().item() <= 2e-2


def test_noalloc_rejects_balanced_split():
    lib = N.load()
    q, kp, vp, bt, seq, mp, npg = _case(13, B=2)
    out = torch.empty_like(q)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    assert _noalloc(q, kp, vp, bt, seq, mp, npg, 0, out, status) == -1
    assert b"balanced" in lib.llmc_last_error_string()
