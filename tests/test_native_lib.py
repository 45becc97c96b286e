"""CPU checks of the C ABI boundary: the library loads, exports every symbol the
header declares, and rejects bad arguments on the host before any launch."""

import ctypes
import os
import re

import pytest
import torch

import llm_cuda_b200._native as N
from llm_cuda_b200.kernels.decode_attention import (
    can_use_triton_decode_attention,
    choose_partition_tokens,
)

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    names = set()
    inc = os.path.join(ROOT, "include")
    for f in os.listdir(inc):
        if f.endswith(".h"):
            src = open(os.path.join(inc, f)).read()
            names |= set(re.findall(r"LLMC_API\s+[\w\s\*]+?\b(llmc_\w+)\s*\(", src))
    return names


def test_library_exports_every_declared_symbol():
    lib = N.load()
    declared = _declared_symbols()
    assert declared, "no declarations found"
    assert declared <= set(N.SIGNATURES), "ctypes table misses a declared symbol"
    for name in declared:
        assert hasattr(lib, name), name
    assert b"sm_100a" in lib.llmc_version()


def _declared_param_counts():
    counts = {}
    inc = os.path.join(ROOT, "include")
    for f in os.listdir(inc):
        if f.endswith(".h"):
            src = open(os.path.join(inc, f)).read()
            for name, params in re.findall(r"LLMC_API\s+[\w\s\*]+?\b(llmc_\w+)\s*\(([^)]*)\)",
                                           src):
                params = params.strip()
                counts[name] = 0 if params in ("", "void") else params.count(",") + 1
    return counts


def test_ctypes_signatures_match_header():
    """Every ctypes prototype has as many arguments as the header's declaration."""
    counts = _declared_param_counts()
    assert counts
    for name, n in counts.items():
        assert len(N.SIGNATURES[name][1]) == n, (name, len(N.SIGNATURES[name][1]), n)


def test_host_validation_without_gpu():
    lib = N.load()
    nul = None
    # Hq not a multiple of Hkv
    rc = lib.llmc_paged_decode(1, 1, 1, 1, 1, 1, nul, nul, 1, 1, 5, 3, 64, 16, 4, 8, 256,
                               0.125, N.LLMC_BF16, 0, nul)
    assert rc == -1 and b"multiple" in lib.llmc_last_error_string()
    # partition not a multiple of 64
    rc = lib.llmc_paged_decode(1, 1, 1, 1, 1, 1, nul, nul, 1, 1, 8, 2, 64, 16, 4, 8, 100,
                               0.125, N.LLMC_BF16, 0, nul)
    assert rc == -1 and b"partition" in lib.llmc_last_error_string()
    # head_dim too large
    rc = lib.llmc_paged_decode(1, 1, 1, 1, 1, 1, nul, nul, 1, 1, 8, 2, 512, 16, 4, 8, 256,
                               0.125, N.LLMC_BF16, 0, nul)
    assert rc == -2
    # split-K workspace required
    rc = lib.llmc_paged_decode(1, 1, 1, 1, 1, 1, nul, nul, 1, 1, 8, 2, 64, 16, 64, 8, 256,
                               0.125, N.LLMC_BF16, 0, nul)
    assert rc == -1 and b"part_o" in lib.llmc_last_error_string()
    # bad dtype / odd head_dim for RoPE
    rc = lib.llmc_rope_append(1, 1, 1, 1, 1, 1, 1, 1, nul, nul, 1, 1, 4, 2, 63, 16, 4, 8, 0, 2,
                              1, nul)
    assert rc == -1 and b"even" in lib.llmc_last_error_string()
    rc = lib.llmc_lse_merge(nul, nul, 1, 1, 1, 8, 64, 2, 256, 7, nul)
    assert rc == -1
    # the error string is cleared by a successful call
    assert lib.llmc_num_partitions(4096, 1024) == 4
    sz = ctypes.c_size_t(0)
    assert lib.llmc_decode_partials_bytes(2, 8, 128, 4, ctypes.byref(sz)) == 2 * 8 * 4 * 128 * 4
    assert sz.value == 2 * 8 * 4 * 4


def test_predicate_matches_reference_on_cpu():
    """Reference predicate semantics (decode_attention.py:162-201): CPU inputs -> False."""
    q = torch.randn(1, 4, 1, 16, dtype=torch.float16)
    k = torch.randn(1, 2, 8, 16, dtype=torch.float16)
    assert can_use_triton_decode_attention(q, k, k) is False
    assert can_use_triton_decode_attention(q, k, k, attention_mask=torch.zeros(1)) is False


def test_partition_choice_balances_work():
    # Config 2: 64 x 4096 tokens, 8 KV heads: more than one item per SM, no long tail.
    T = choose_partition_tokens([4096] * 64, 8, 4, 148)
    items = 64 * (4096 // T) * 8
    assert items >= 2 * 148 and 4096 % T == 0
    # one short sequence: a single partition
    assert choose_partition_tokens([80], 2, 4, 148) >= 256
    # empty batch
    assert choose_partition_tokens([0, 0], 8, 4, 148) > 0


def test_missing_library_fails_loudly(monkeypatch):
    monkeypatch.setattr(N, "_lib", None)
    monkeypatch.setattr(N, "_LIB_PATH", "/nonexistent/libllmcuda_b200.so")
    with pytest.raises(N.NativeLibraryError):
        N.load()


def test_host_validation_of_step_entry_points():
    """The config-5 step entry points reject bad arguments before touching CUDA."""
    lib = N.load()
    nul = None
    # fused all-reduce: world out of range, rank >= world, rows > rows_cap
    rc = lib.llmc_allreduce_add_rmsnorm(1, 1, 1, 1, 1, 1, 1, 1, 0, 9, 64, 64, 4096, 1e-5,
                                        N.LLMC_BF16, nul)
    assert rc == -1 and b"world" in lib.llmc_last_error_string()
    rc = lib.llmc_allreduce_add_rmsnorm(1, 1, 1, 1, 1, 1, 1, 1, 2, 2, 64, 64, 4096, 1e-5,
                                        N.LLMC_BF16, nul)
    assert rc == -1
    rc = lib.llmc_allreduce_add_rmsnorm(1, 1, 1, 1, 1, 1, 1, 1, 0, 2, 65, 64, 4096, 1e-5,
                                        N.LLMC_BF16, nul)
    assert rc == -1 and b"rows_cap" in lib.llmc_last_error_string()
    # misaligned tensors
    rc = lib.llmc_allreduce_add_rmsnorm(18, 16, 16, 16, 16, 16, 16, 16, 0, 2, 8, 64, 4096,
                                        1e-5, N.LLMC_BF16, nul)
    assert rc == -1 and b"aligned" in lib.llmc_last_error_string()
    fb = ctypes.c_size_t(0)
    # 8-byte words, each carrying 4 bytes of a row: the larger of the one-shot layout
    # (2 parities x world x rows) and the two-shot one (reduce-scatter slices plus
    # all-gather slices with one extra word each)
    w = 4096 * 2 // 4
    for world in (2, 4, 8):
        one = 2 * world * 64 * w
        two = 2 * 64 * w + 2 * world * 64 * (w // world + 1)
        assert lib.llmc_ar_region_bytes(world, 64, 4096, N.LLMC_BF16, ctypes.byref(fb)) == \
            max(one, two) * 8
    assert fb.value == 0
    # argmax
    assert lib.llmc_argmax(1, 1, 70000, 10, N.LLMC_BF16, 8, nul) == -1
    assert lib.llmc_argmax(1, 1, 4, 10, N.LLMC_BF16, 4, nul) == -1        # misaligned workspace
    assert lib.llmc_argmax_workspace_bytes(64) == 64 * 12
    # strided fused step: a sequence stride smaller than the dense one
    args = [1] * 10 + [128] + [1] * 5 + [4, 32, 8, 128, 16, 16, 1024, 0]
    rc = lib.llmc_rope_append_decode_strided(*args, 0.1, N.LLMC_BF16, 32 * 128 - 1, 8 * 128, 0,
                                             nul)
    assert rc == -1 and b"stride" in lib.llmc_last_error_string()
    # decode GEMM shapes
    assert lib.llmc_decode_gemm(1, 1, 1, 1, 4, 1, 64, 100, 64, 1, nul) == -2
    assert lib.llmc_decode_gemm_workspace_bytes(300, 128, 64) == 0
