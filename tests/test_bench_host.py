"""Host-side pieces of bench.py (no GPU): workloads, the config both arms print, the
split-K partial count of the balanced split, and the reference's own CPU decode path
that the reference arm times."""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402
from refsrc import reference_path  # noqa: E402


@pytest.mark.parametrize("world", [1, 2, 8])
def test_weak_scaling_workload_and_config(world):
    w, lengths = bench._workload("c2", "weak", world)
    assert w["B"] == 64 * world and len(lengths) == 64 * world and set(lengths) == {4096}
    cfg = bench._config(w, lengths, world)
    assert cfg["global_batch"] == 64 * world and cfg["parallelism"].startswith(f"tp{world}")
    # every rank streams the same bytes as at N=1
    assert bench._plan(w, lengths, world)["kv_bytes_rank"] == 64 * 4096 * 8 * 128 * 4
    ws, ls = bench._workload("c2", "strong", world)
    assert ws["B"] == 64 and len(ls) == 64


def test_ragged_and_long_workloads():
    w3, l3 = bench._workload("c3", "weak", 1)
    assert len(l3) == 256 and min(l3) >= 128 and max(l3) <= 32768
    assert l3 == bench._workload("c3", "weak", 1)[1]           # seeded
    w4, l4 = bench._workload("c4", "weak", 1)
    assert l4 == [131072] * 4 and w4["part"] == 4096


def _partials_brute(lengths, hkv, group, grid):
    hg = (group + 7) // 8
    rows = [((L + 63) // 64, min(8, group - 8 * j)) for L in lengths for _ in range(hkv)
            for j in range(hg)]
    total = sum(c for c, _ in rows)
    starts = [c * total // grid for c in range(grid + 1)]
    owner = []
    for c in range(grid):
        owner += [c] * (starts[c + 1] - starts[c])
    n, x = 0, 0
    for chunks, heads in rows:
        if chunks:
            segs = len(set(owner[x:x + chunks]))
            if segs > 1:
                n += segs * heads
        x += chunks
    return n


@pytest.mark.parametrize("lengths,hkv,group,grid", [
    ([4096] * 64, 8, 4, 148), ([100], 8, 1, 148), ([300, 40, 1, 0, 2049], 2, 12, 7),
    ([131072] * 4, 8, 8, 148)])
def test_balanced_partials_count(lengths, hkv, group, grid):
    assert bench._balanced_partials(lengths, hkv, group, grid) == \
        _partials_brute(lengths, hkv, group, grid)


def test_merge_clocks():
    a = {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": [], "samples": 3, "power_w_max": 500}
    b = {"sm_mhz": 1800.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 2,
         "power_w_max": 900}
    m = bench._merge_clocks([a, None, b, {"samples": 0}])
    assert m["reasons"] == ["sw_power_cap"] and m["samples"] == 5 and m["power_w_max"] == 900
    assert bench._merge_clocks([])["reasons"] == ["unavailable"]


@pytest.mark.skipif(reference_path() is None, reason="reference not installed in baseline/_ref")
def test_reference_cpu_path_runs_the_reference_code():
    w = dict(B=3, Hq=4, Hkv=2, d=16, P=4, scale=1.0, part=None, seed=7, scaling="weak")
    path = bench.ReferenceCpuPath(w, [9, 13, 5])
    assert len(path.pool) == 3
    assert path.step() == 9 * 2 * 16 * 2 * 2        # the whole context's K and V, bf16
    assert path.step() == 13 * 2 * 16 * 2 * 2
    assert path.pool[0].length == 8                  # rolled back: the next call re-appends
    assert type(path.pool[0]).__module__.startswith("llm_cuda.")   # the reference's class
