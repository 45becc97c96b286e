"""Host-side check of the fused all-reduce's shared-region layout (no GPU needed).

The one-shot and two-shot kernels (``csrc/allreduce.cu``) address each rank's region
as 8-byte words.  This test replays their word indices for every (rank, row, vector,
word) of both algorithms and both parities, over a region of the size the library
reports (``llmc_ar_region_bytes``), and checks that every word lands inside the
region, that no two senders write the same word, and that every receiver reads exactly
the words its sender wrote.  (The 2-rank two-shot layout once overran a region sized
for the one-shot layout only.)
"""

import ctypes

import numpy as np
import pytest

from llm_cuda_b200 import _native as N


def _region_words(world, rows_cap, hidden, dt=N.LLMC_BF16):
    fb = ctypes.c_size_t(0)
    b = N.load().llmc_ar_region_bytes(world, rows_cap, hidden, dt, ctypes.byref(fb))
    assert fb.value == 0 and b % 8 == 0
    return b // 8


def _one_shot(world, rows_cap, nvec):
    """(dest rank, word) written for (src, par, b, i, j), and the word the dest reads."""
    row_words = 4 * nvec
    slot = world * rows_cap * row_words
    for par in (0, 1):
        for src in range(world):
            for dst in range(world):
                if dst == src:
                    continue
                for b in range(rows_cap):
                    base = par * slot + (src * rows_cap + b) * row_words
                    for i in range(nvec):
                        for j in range(4):
                            w = base + j * nvec + i
                            # receiver dst reads src's word j of vector i of row b here
                            r = par * slot + ((src * rows_cap + b) * row_words + i) + j * nvec
                            yield dst, w, r, (src, par, b, i, j)


def _two_shot(world, rows_cap, nvec):
    nvs = nvec // world
    sw = 4 * nvs
    rs_par = world * rows_cap * sw
    ag_base = 2 * rs_par
    ag_par = world * rows_cap * (sw + 1)
    for par in (0, 1):
        for src in range(world):
            for b in range(rows_cap):
                for i in range(nvec):
                    q, li = divmod(i, nvs)
                    for j in range(4):
                        # reduce-scatter: src -> owner q
                        if q != src:
                            w = par * rs_par + (src * rows_cap + b) * sw + li + j * nvs
                            r = par * rs_par + (src * rows_cap + b) * sw + li + j * nvs
                            yield q, w, r, ("rs", src, par, b, i, j)
                        # all-gather: owner src -> every other rank
                        if q == src:
                            for dst in range(world):
                                if dst == src:
                                    continue
                                w = ag_base + par * ag_par + (src * rows_cap + b) * (sw + 1) + li + j * nvs
                                r = ag_base + par * ag_par + (q * rows_cap + b) * (sw + 1) + li + j * nvs
                                yield dst, w, r, ("ag", src, par, b, i, j)
                for dst in range(world):   # the slice's sum of squares
                    if dst != src:
                        w = ag_base + par * ag_par + (src * rows_cap + b) * (sw + 1) + sw
                        yield dst, w, w, ("ss", src, par, b)


@pytest.mark.parametrize("algo", ["one_shot", "two_shot"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_region_layout(world, algo):
    rows_cap, hidden = 3, 4096 if world == 8 else 1024        # bf16: 8 elements per vector
    nvec = hidden // 8
    words = _region_words(world, rows_cap, hidden)
    gen = _one_shot if algo == "one_shot" else _two_shot
    seen = [dict() for _ in range(world)]
    for dst, w, r, tag in gen(world, rows_cap, nvec):
        assert 0 <= w < words, (tag, w, words)
        assert w == r, tag                          # the receiver reads what was written
        assert w not in seen[dst], (tag, seen[dst].get(w))
        seen[dst][w] = tag
    # every rank receives the same number of words
    assert len({len(x) for x in seen}) == 1
