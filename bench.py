"""Decode-attention benchmark (driver contract: one JSON line from rank 0).

A step is one pass of the hot path over one batch: fused RoPE + KV-page append of
the new token of every sequence, paged GQA flash-decode over the whole context,
and the split-K log-sum-exp merge.  Default workload = BASELINE config 2
(Llama-3-8B decode attention: B64 Hq32 Hkv8 d128, context 4096, page 16,
shuffled block tables, bf16).

Under torchrun with N ranks the decode-attention step is KV-head sharded (each rank
owns Hkv/N KV heads and their query heads, as the reference's column split of
q/k/v_proj).  By default the scaling is WEAK: N x the config's batch, so every rank
streams the same bytes as at N=1 and `value` stays comparable across N; this path
has no data-path collective.  `--scaling strong` splits the config's own batch.

The same line also carries, at every N:
  * ``c5``: the config-5 full decode step (32-layer Llama-3-8B shape, B=64, KV
    prefilled to 2048) at TP=N: tokens/s with the fused NVLink all-reduce and with
    NCCL, HBM fraction per GPU, the per-phase split of a step, and (N>1) the logits
    of TP=N against a TP1 model on rank 0;
  * at N=1: ``c3``/``c4`` sub-results, the reference's own Triton kernel on this GPU
    (``reference_gpu_kernel``) and ``cpu_baseline`` (the reference's torch CPU path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c2|c3|c4|c5] [--scaling weak|strong] [--no-extras]

``--impl reference`` times the reference's own CPU implementation of the path (its
torch code from ``baseline/_ref``: ``apply_rotary`` fallback, ``PagedKVLayerCache``
append + ``get_kv``, ``_repeat_kv`` + ``_torch_attention``) on the host cores; under
torchrun only rank 0 runs it.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import platform
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L2_BYTES = 126 * 1024 * 1024
THETA = 500000.0
REF_DIR = os.path.join(ROOT, "baseline", "_ref")

WORKLOADS = {
    "c2": dict(B=64, Hq=32, Hkv=8, d=128, P=16, scale=1.0, part=None, seed=1002,
               desc="config2 Llama-3-8B decode-attention step: B64 Hq32 Hkv8 d128 ctx4096 page16 "
                    "shuffled block tables"),
    "c3": dict(B=256, Hq=32, Hkv=8, d=128, P=16, scale=1.0, part=None, seed=1003,
               desc="config3 ragged batch: B256 Hq32 Hkv8 d128 ctx~U[128,32768] page16 shared pool"),
    "c4": dict(B=4, Hq=64, Hkv=8, d=128, P=64, scale=0.5, part=4096, seed=1004,
               desc="config4 long context split-K: B4 Hq64 Hkv8 d128 ctx131072 page64 "
                    "4096-token partitions + LSE merge"),
}


def _lengths(name: str, w: dict) -> list[int]:
    if name == "c2":
        return [4096] * w["B"]
    if name == "c3":
        g = torch.Generator().manual_seed(w["seed"])
        return torch.randint(128, 32769, (w["B"],), generator=g).tolist()
    return [131072] * w["B"]


def _workload(name: str, scaling: str, world: int) -> tuple[dict, list[int]]:
    w = dict(WORKLOADS[name])
    w["scaling"] = scaling
    if scaling == "weak" and world > 1:
        # Weak scaling: the config's batch per GPU, N times the sequences in all,
        # every rank holding its 1/N of the KV heads of all of them.
        w["B"] *= world
        w["desc"] += f" (global batch {w['B']} = {world} x the config's, weak scaling)"
    return w, _lengths(name, w)


def _peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        return {"hbm_gbs": float(pk["hbm_gbs"]), "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "source": "fallback"}


def _profile_traffic(workload: str, n_gpus: int):
    """dram bytes per decode launch from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", f"paged_decode_{workload}_traffic.json")
    try:
        with open(path) as f:
            rec = json.load(f)
        return rec.get(f"tp{n_gpus}")
    except Exception:
        return None


def _host_info() -> dict:
    model = platform.processor() or ""
    try:
        out = subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout
        for line in out.splitlines():
            if line.startswith("Model name:"):
                model = line.split(":", 1)[1].strip()
    except Exception:
        pass
    return {"nproc": os.cpu_count(), "cpu_model": model}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.idx)],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        try:
            for line in open(self.path):
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                    rows.append(parts)
        except Exception:
            pass
        finally:
            if self.path and os.path.exists(self.path):
                os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        sm = [float(r[1]) for r in rows]
        mx = max(float(r[2]) for r in rows)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows)}


def _merge_clocks(parts: list[dict]) -> dict:
    """One clocks record over several sampled regions (median of medians, union of
    reasons)."""
    parts = [c for c in parts if c and c.get("samples")]
    if not parts:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
    return {"sm_mhz": statistics.median(c["sm_mhz"] for c in parts),
            "sm_max_mhz": max(c["sm_max_mhz"] for c in parts),
            "reasons": sorted({r for c in parts for r in c["reasons"]}),
            "samples": sum(c["samples"] for c in parts),
            "power_w_max": max(c.get("power_w_max", 0.0) for c in parts)}


# ---------------------------------------------------------------------------
# CPU baselines
# ---------------------------------------------------------------------------
def _import_reference():
    """The unmodified reference package from baseline/_ref, or None."""
    if not os.path.isdir(os.path.join(REF_DIR, "llm_cuda")):
        return None
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import llm_cuda

    return llm_cuda


class ReferenceCpuPath:
    """The reference's own CPU decode-attention path for one sequence per call, run
    exactly as its ``Llama3Attention.forward`` decode branch does on the CPU
    (``attention.py:104-147`` of llm-cuda): ``build_rope_cache`` + ``apply_rotary``
    (the torch branch, ``rotary.py:29-109``), ``PagedKVLayerCache.append`` +
    ``get_kv`` (``kv_cache.py:38-83``; the reference cache holds one sequence), then
    ``_repeat_kv`` + ``_torch_attention`` (``attention.py:56-89``).  A pool of distinct
    seeded sequences (each its own reference cache) is cycled, with a fresh q/k/v for
    every call, so no call finds its K/V in the CPU caches of the previous one."""

    def __init__(self, w: dict, lengths: list[int], dtype=torch.bfloat16,
                 pool_bytes: int = 256 << 20):
        ref = _import_reference()
        if ref is None:
            raise RuntimeError("reference not installed in baseline/_ref")
        from llm_cuda.models.llama3.attention import Llama3Attention
        from llm_cuda.models.llama3.config import Llama3Config
        from llm_cuda.models.llama3.kv_cache import PagedKVLayerCache
        from llm_cuda.models.llama3.rotary import apply_rotary, build_rope_cache

        torch.set_num_threads(os.cpu_count())
        self.apply_rotary, self.build_rope_cache = apply_rotary, build_rope_cache
        Hq, Hkv, d, P = w["Hq"], w["Hkv"], w["d"], w["P"]
        self.Hq, self.Hkv, self.d, self.dtype = Hq, Hkv, d, dtype
        self.att = Llama3Attention(Llama3Config(hidden_size=Hq * d, num_attention_heads=Hq,
                                                num_key_value_heads=Hkv, num_hidden_layers=1,
                                                intermediate_size=256, vocab_size=8))
        seq_bytes = max(lengths) * Hkv * d * 2 * 2
        n_pool = max(1, min(8, pool_bytes // max(1, seq_bytes), len(lengths)))
        g = torch.Generator().manual_seed(w["seed"] + 4242)
        self.pool = []
        for i in range(n_pool):
            L = lengths[i]
            c = PagedKVLayerCache(Hkv, d, L, P, torch.device("cpu"), dtype)
            c.key_pages.copy_(torch.randn(c.key_pages.shape, generator=g) * w["scale"])
            c.value_pages.copy_(torch.randn(c.value_pages.shape, generator=g) * w["scale"])
            c.length = L - 1                      # the new token goes to position L-1
            self.pool.append(c)
        self.g = g
        self.scale = w["scale"]
        self.i = 0

    def step(self) -> int:
        """One sequence's decode-attention step; returns its K/V bytes."""
        c = self.pool[self.i % len(self.pool)]
        self.i += 1
        g, s = self.g, self.scale
        q = (torch.randn(1, self.Hq, 1, self.d, generator=g) * s).to(self.dtype)
        k = (torch.randn(1, self.Hkv, 1, self.d, generator=g) * s).to(self.dtype)
        v = (torch.randn(1, self.Hkv, 1, self.d, generator=g) * s).to(self.dtype)
        pos = c.length
        cos, sin = self.build_rope_cache(seq_len=1, head_dim=self.d, base=THETA,
                                         device=q.device, dtype=q.dtype, position_offset=pos,
                                         inv_freq=self.att.inv_freq)
        q, k = self.apply_rotary(q, k, cos, sin)
        c.append(k, v)
        kk, vv = c.get_kv()
        self.att._torch_attention(q, self.att._repeat_kv(kk), self.att._repeat_kv(vv),
                                  attention_mask=None, past_len=pos)
        c.length = pos                            # the next call appends at the same slot
        return (pos + 1) * self.Hkv * self.d * 2 * 2


def _port_unit(rng, L, G, d, dt):
    from oracle import decode_oracle as O

    q = O.round_to(rng.standard_normal((G, d), dtype=np.float32), dt)
    k = O.round_to(rng.standard_normal((1, L, d), dtype=np.float32), dt)
    v = O.round_to(rng.standard_normal((1, L, d), dtype=np.float32), dt)
    cos, sin = O.build_rope_cache([L - 1], d, THETA, dt)
    return q, k, v, cos, sin


def port_cpu_baseline(w: dict, lengths, budget_s: float) -> dict:
    """Secondary CPU figure: the numpy oracle restatement on (sequence, KV head) units
    (distinct seeded units from a pool, cycled)."""
    from oracle import decode_oracle as O

    dt = "bf16"
    G, d = w["Hq"] // w["Hkv"], w["d"]
    rng = np.random.default_rng(0)
    L = int(lengths[len(lengths) // 2])
    pool = [_port_unit(rng, L, G, d, dt) for _ in range(8)]
    n, kv_bytes = 0, 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        q, k, v, cos, sin = pool[n % len(pool)]
        O.decode_attention(O.apply_rotary(q[:, None], cos, sin, dt)[:, 0], k, v, dt)
        n += 1
        kv_bytes += L * d * 2 * 2
    el = time.perf_counter() - t0
    return {"value": kv_bytes / el / 1e9, "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{n} (sequence, KV head) units of ctx {L} from a pool of 8, {el:.1f} s "
                      "(numpy oracle restatement, OpenBLAS threads)"}


def reference_cpu_baseline(w: dict, lengths, budget_s: float) -> dict:
    """The reference's own torch CPU path timed for ~budget_s on distinct sequences."""
    path = ReferenceCpuPath(w, lengths)
    path.step()                                    # warm (allocator, thread pool)
    n, kv = 0, 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        kv += path.step()
        n += 1
    el = time.perf_counter() - t0
    hi = _host_info()
    return {"value": kv / el / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": "reference", "nproc": hi["nproc"], "cpu_model": hi["cpu_model"],
            "sample": f"{n} full sequences (all {w['Hkv']} KV / {w['Hq']} query heads) at ctx "
                      f"{lengths[0]}, cycling {len(path.pool)} distinct seeded caches, "
                      f"{el:.1f} s; the reference's torch CPU decode branch from baseline/_ref "
                      f"(attention.py:104-147 with rotary.py:104-109, kv_cache.py:38-83), "
                      f"torch threads {torch.get_num_threads()}"}


def run_reference(args, name, w, lengths, config):
    """--impl reference: the reference's CPU path on this host's cores (rank 0 only)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    try:
        path = ReferenceCpuPath(w, lengths)
        kind = "reference"
    except Exception as e:   # the package is missing: the oracle port stands in
        path, kind, why = None, "port", f"{type(e).__name__}: {e}"
    if path is None:
        rng = np.random.default_rng(0)
        G, d = w["Hq"] // w["Hkv"], w["d"]
        L = int(lengths[len(lengths) // 2])
        pool = [_port_unit(rng, L, G, d, "bf16") for _ in range(8)]
        from oracle import decode_oracle as O

        state = {"i": 0}

        def one():
            q, k, v, cos, sin = pool[state["i"] % len(pool)]
            state["i"] += 1
            O.decode_attention(O.apply_rotary(q[:, None], cos, sin, "bf16")[:, 0], k, v, "bf16")
            return L * d * 2 * 2
    else:
        one = path.step
    one()
    t0 = time.perf_counter()
    one()
    t_unit = max(time.perf_counter() - t0, 1e-4)
    budget = 150.0 / max(1, args.steps + args.warmup)
    units = max(1, int(budget / t_unit))
    for _ in range(args.warmup):
        for _ in range(units):
            one()
    kv = 0
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for _ in range(units):
            kv += one()
    el = time.perf_counter() - t0
    value = kv / el / 1e9
    hi = _host_info()
    unit_desc = ("full sequences (all KV / query heads)" if kind == "reference" else
                 "(sequence, KV head) units of the numpy port (" + why + ")")
    line = {
        "impl": "reference", "metric": "decode-attn KV GB/s", "value": value, "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3,
        "higher_is_better": True, "scaling": w["scaling"], "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) K/V, fresh q/k/v per call)", "config": config,
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": torch.get_num_threads(),
                         "kind": kind, "nproc": hi["nproc"], "cpu_model": hi["cpu_model"],
                         "sample": f"{units} {unit_desc} per step, ctx {lengths[0]}"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def _dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def _barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def _max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def triton_reference_compare(st, lengths) -> dict:
    """Time the reference's own GPU kernel, ``triton_decode_attention``
    (``src/llm_cuda/kernels/triton/decode_attention.py:204-287`` of llm-cuda,
    installed unmodified in ``baseline/_ref``), on this step's data.  It needs dense
    ``[B, Hkv, L, d]`` K/V, so the pages are gathered first (the reference's
    ``get_kv``, ``kv_cache.py:65-83``, does the same copy each step); the gather is
    timed separately."""
    if _import_reference() is None:
        return {"unavailable": "baseline/_ref not installed"}
    if len(set(lengths)) != 1:
        return {"unavailable": "ragged batch: the reference kernel takes one kv_len"}
    # The unmodified reference kernel reads a module-level float inside @triton.jit,
    # which Triton 3.6 rejects unless this documented Triton switch is set.
    os.environ.setdefault("TRITON_ALLOW_NON_CONSTEXPR_GLOBALS", "1")
    from llm_cuda.kernels.triton.decode_attention import triton_decode_attention as ref_decode

    c = st["cache"]
    L = lengths[0]
    n = math.ceil(L / c.page_size)
    idx = c.block_table[:, :n].long()

    def gather(pages):
        g = pages[idx].permute(0, 2, 1, 3, 4).reshape(c.batch_size, c.num_kv_heads,
                                                      n * c.page_size, c.head_dim)
        return g[:, :, :L].contiguous()

    q = st["q_rot"]
    k, v = gather(c.key_pages), gather(c.value_pages)
    out_ref = ref_decode(q, k, v)
    torch.cuda.synchronize()
    times = {}
    for name, fn in (("gather_ms", lambda: (gather(c.key_pages), gather(c.value_pages))),
                     ("kernel_ms", lambda: ref_decode(q, k, v))):
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(20):
            fn()
        e1.record()
        torch.cuda.synchronize()
        times[name] = e0.elapsed_time(e1) / 20
    kv = sum(lengths) * c.num_kv_heads * c.head_dim * 4
    ours = st["out"].float()
    return {"kernel": "llm_cuda triton_decode_attention (baseline/_ref, Triton JIT for sm_100)",
            "kernel_ms": times["kernel_ms"], "gather_ms": times["gather_ms"],
            "kv_gbs_kernel_only": kv / (times["kernel_ms"] * 1e-3) / 1e9,
            "kv_gbs_with_gather": kv / ((times["kernel_ms"] + times["gather_ms"]) * 1e-3) / 1e9,
            "max_abs_diff_vs_ours": (out_ref[:, :, 0].float() - ours).abs().max().item()}


def _balanced_partials(lengths, hkv: int, group: int, grid: int) -> int:
    """Split-K partials (one per query head and segment) that the balanced split writes
    and the merge reads back: rows (sequence, KV head, head group) of ceil(L/64)
    chunks laid end to end, CTA c taking chunks [c*total/grid, (c+1)*total/grid)."""
    hg = (group + 7) // 8
    chunks = [(L + 63) // 64 for L in lengths for _ in range(hkv * hg)]
    heads = [min(8, group - 8 * j) for _ in lengths for _ in range(hkv) for j in range(hg)]
    total = sum(chunks)
    if total == 0:
        return 0

    def owner(x):
        return ((x + 1) * grid + total - 1) // total - 1

    n, x0 = 0, 0
    for c, h in zip(chunks, heads):
        if c:
            if total >= grid:   # every CTA owns a chunk: the owners are consecutive
                segs = owner(x0 + c - 1) - owner(x0) + 1
            else:               # some CTAs own nothing and hold no segment
                segs = len({owner(x) for x in range(x0, x0 + c)})
            if segs > 1:
                n += segs * h
        x0 += c
    return n


def _plan(w: dict, lengths, world: int) -> dict:
    hkv, hq = w["Hkv"] // world, w["Hq"] // world
    kv_bytes_rank = sum(lengths) * hkv * w["d"] * 2 * 2
    n_sets = max(1, math.ceil(3 * L2_BYTES / kv_bytes_rank)) if kv_bytes_rank < 3 * L2_BYTES else 1
    return dict(hkv=hkv, hq=hq, kv_bytes_rank=kv_bytes_rank, n_sets=n_sets)


def _config(w: dict, lengths, world: int) -> dict:
    pl = _plan(w, lengths, world)
    T = w["part"]
    return {"workload": w["desc"], "B": w["B"], "global_batch": w["B"], "Hq": w["Hq"],
            "Hkv": w["Hkv"], "head_dim": w["d"], "page_size": w["P"],
            "context_tokens_total": sum(lengths),
            "partition_tokens": T if T else "balanced",
            "parallelism": f"tp{world} (KV-head sharded)", "input_sets": pl["n_sets"],
            "l2": f"KV per rank {pl['kv_bytes_rank'] / 1e6:.0f} MB x {pl['n_sets']} rotating "
                  f"sets > L2 126 MB (no flush needed)",
            "graph": "each step replayed from a CUDA graph"}


def measure_decode(name: str, w: dict, lengths, steps: int, warmup: int, world: int,
                   rank: int, dev, with_e2e: bool = True, with_triton: bool = False) -> dict:
    """Time the fused decode-attention step of workload ``name`` on this rank's KV-head
    shard: K graph replays (device time, max over ranks), the decode kernel's own
    duration inside the graph, and the public graphed step with host buffers (e2e)."""
    from llm_cuda_b200.kernels.decode_attention import BALANCED, rope_append_decode
    from llm_cuda_b200.models.llama3 import PagedKVLayerCache, RopeTable, make_block_table
    from llm_cuda_b200.models.llama3.kv_cache import GraphedDecodeStep

    B, Hq, Hkv, d, P = w["B"], w["Hq"], w["Hkv"], w["d"], w["P"]
    if Hkv % world:
        raise SystemExit(f"KV heads {Hkv} do not shard over {world} ranks")
    pl = _plan(w, lengths, world)
    hkv, hq, kv_bytes_rank, n_sets = pl["hkv"], pl["hq"], pl["kv_bytes_rank"], pl["n_sets"]
    dtype = torch.bfloat16
    pages_per = [math.ceil(L / P) for L in lengths]
    max_pages = max(pages_per)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    # Configs 2/3: the balanced split (equal chunk ranges per SM, computed on the
    # device); config 4 names its 4096-token partitions.
    T = w["part"] or BALANCED

    gen = torch.Generator().manual_seed(w["seed"] + 7919 * rank)
    gd = torch.Generator(device=dev).manual_seed(w["seed"] + rank)
    rope = RopeTable(max_pages * P, d, THETA, dev, dtype)
    sets = []
    for s in range(n_sets):
        num_pages = sum(pages_per) + 8
        bt = make_block_table(B, pages_per, num_pages, max_pages, generator=gen)
        cache = PagedKVLayerCache(hkv, d, max_pages * P, P, dev, dtype, batch_size=B,
                                  num_pages=num_pages, block_table=bt)
        cache.key_pages.normal_(generator=gd).mul_(w["scale"])
        cache.value_pages.normal_(generator=gd).mul_(w["scale"])
        base = torch.tensor([L - 1 for L in lengths], dtype=torch.int32, device=dev)
        q = (torch.randn(B, hq, 1, d, device=dev, generator=gd) * w["scale"]).to(dtype)
        k = (torch.randn(B, hkv, 1, d, device=dev, generator=gd) * w["scale"]).to(dtype)
        v = (torch.randn(B, hkv, 1, d, device=dev, generator=gd) * w["scale"]).to(dtype)
        sets.append(dict(cache=cache, base=base, q=q, k=k, v=v, q_rot=torch.empty_like(q),
                         out=torch.empty(B, hq, d, device=dev, dtype=dtype)))
    base_host = [L - 1 for L in lengths]

    def step(st, ev=None):
        # One fused launch does RoPE on the new token, the page append and the paged
        # attention (and, with the balanced split, the merge and the length update).
        c = st["cache"]
        c.seq_lens.copy_(st["base"])          # every step attends exactly the configured context
        c.host_lengths = list(base_host)
        rope_append_decode(st["q"], st["k"], st["v"], c.key_pages, c.value_pages,
                           c.block_table, c.seq_lens, rope.cos, rope.sin, host_lens=base_host,
                           partition_tokens=T, out=st["out"], q_out=st["q_rot"],
                           workspace=c.workspace, status=c.status, events=ev)

    for st in sets:                           # eager warm-up: workspaces exist before capture
        step(st)
    torch.cuda.synchronize()
    for st in sets:
        st["cache"].check_status()

    def capture(fn):
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                fn()
        torch.cuda.current_stream(dev).wait_stream(s)
        return g

    graphs = [capture(lambda st=st: step(st)) for st in sets]
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for i in range(max(3, warmup)):
            graphs[i % n_sets].replay()
    torch.cuda.synchronize()
    _barrier(world)

    clock = ClockSampler(dev.index if world > 1 else 0)
    with clock:
        # ---- timed region: K graph replays ----
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        _barrier(world)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("decode_steps")
        with torch.cuda.stream(stream):
            e0.record(stream)
            for i in range(steps):
                graphs[i % n_sets].replay()
            e1.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        _barrier(world)
        ms = e0.elapsed_time(e1) / steps
        # ---- the decode kernel's duration inside the graph: copies of the step graph
        # with timing event nodes around the decode launch (the length reset sits
        # before the first node), one event pair per copy, replayed back to back as in
        # the timed loop and read after one synchronisation ----
        kreps = 24
        try:
            evs = [(torch.cuda.Event(enable_timing=True, external=True),
                    torch.cuda.Event(enable_timing=True, external=True)) for _ in range(kreps)]
            tg = [capture(lambda st=sets[j % n_sets], ev=evs[j]: step(st, ev))
                  for j in range(kreps)]
            torch.cuda.synchronize()
            times = []
            for _ in range(3):                     # the last round is the one read
                with torch.cuda.stream(stream):
                    for g in tg:
                        g.replay()
                torch.cuda.synchronize()
                times = [a.elapsed_time(b) for a, b in evs]
            k_ms = statistics.mean(times)
            k_how = ("in-graph: copies of the step graph with timing event nodes around the "
                     "decode launch, replayed back to back")
            del tg
        except Exception as ex:   # timing nodes unsupported: eager launches instead
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(kreps)]
            with torch.cuda.stream(stream):
                for i in range(kreps):
                    torch.cuda._sleep(200_000)
                    step(sets[i % n_sets], evs[i])
            torch.cuda.synchronize()
            k_ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
            k_how = f"cold_isolated eager launches ({type(ex).__name__})"
    clocks = clock.summary()
    for st in sets:
        st["cache"].check_status()
    tri = None
    if with_triton and rank == 0:
        try:
            tri = triton_reference_compare(sets[0], lengths)
        except Exception as e:  # informative only; never fails the bench line
            tri = {"unavailable": f"{type(e).__name__}: {str(e)[:200]}"}
    ms = _max_over_ranks(ms, world)
    k_ms = _max_over_ranks(k_ms, world)

    e2e = None
    if with_e2e:
        st = sets[0]
        c = st["cache"]
        # The step's host inputs (new token's q, k, v) packed in one pinned buffer: one
        # H2D copy per step into one of two device buffers, on a copy stream, so the
        # transfers of step i+1 and the D2H read of step i's output overlap step i's
        # compute; events order the buffers.
        nq, nk = B * hq * d, B * hkv * d
        h_in = torch.empty(nq + 2 * nk, dtype=dtype, pin_memory=True)
        h_in[:nq].copy_(st["q"].reshape(-1).cpu())
        h_in[nq:nq + nk].copy_(st["k"].reshape(-1).cpu())
        h_in[nq + nk:].copy_(st["v"].reshape(-1).cpu())
        h_out = [torch.empty(B, hq, 1, d, dtype=dtype, pin_memory=True) for _ in range(2)]
        d_in = [torch.empty(nq + 2 * nk, dtype=dtype, device=dev) for _ in range(2)]
        c.seq_lens.copy_(st["base"])
        c.host_lengths = list(base_host)
        steps_g = [GraphedDecodeStep(c, rope, d_in[j][:nq].view(B, hq, 1, d),
                                     d_in[j][nq:nq + nk].view(B, hkv, 1, d),
                                     d_in[j][nq + nk:].view(B, hkv, 1, d), partition_tokens=T)
                   for j in range(2)]
        d_out = [g.out for g in steps_g]
        copy_s = torch.cuda.Stream(device=dev)
        main_s = torch.cuda.current_stream(dev)
        in_ready = [torch.cuda.Event() for _ in range(2)]
        in_free = [torch.cuda.Event() for _ in range(2)]
        out_ready = [torch.cuda.Event() for _ in range(2)]
        out_free = [torch.cuda.Event() for _ in range(2)]
        for e in in_free + out_free:
            e.record(main_s)
        e2e_steps = max(10, min(steps, 500))
        _barrier(world)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for i in range(e2e_steps + 1):
            j = i % 2
            if i < e2e_steps:                       # H2D of step i
                copy_s.wait_event(in_free[j])
                with torch.cuda.stream(copy_s):
                    d_in[j].copy_(h_in, non_blocking=True)
                in_ready[j].record(copy_s)
            if i >= 1:                              # D2H of step i-1
                jp = (i - 1) % 2
                copy_s.wait_event(out_ready[jp])
                with torch.cuda.stream(copy_s):
                    h_out[jp].view(B, hq, d).copy_(d_out[jp], non_blocking=True)
                out_free[jp].record(copy_s)
            if i < e2e_steps:                       # compute of step i
                main_s.wait_event(in_ready[j])
                main_s.wait_event(out_free[j])
                c.seq_lens.copy_(st["base"])
                c.host_lengths = list(base_host)
                steps_g[j].replay()
                in_free[j].record(main_s)
                out_ready[j].record(main_s)
        torch.cuda.synchronize()
        e2e_ms = (time.perf_counter() - t0) / e2e_steps * 1e3
        _barrier(world)
        e2e_ms = _max_over_ranks(e2e_ms, world)
        total_kv = sum(lengths) * Hkv * d * 2 * 2
        e2e = {"value": total_kv / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
               "ms_per_step": e2e_ms, "tokens_per_s": B / (e2e_ms * 1e-3),
               "h2d_bytes_per_step": h_in.numel() * h_in.element_size(),
               "d2h_bytes_per_step": h_out[0].numel() * h_out[0].element_size(),
               "path": "GraphedDecodeStep (the fused RoPE+append+decode step, one graph "
                       "launch per step) with pinned host in/out, copies on a second "
                       "stream overlapping compute"}
        del steps_g

    total_kv = sum(lengths) * Hkv * d * 2 * 2         # all ranks together
    value = total_kv / (ms * 1e-3) / 1e9
    # algorithmic bytes of the fused decode launch (+ the merge launch with uniform
    # partitions) on one rank: K/V of the whole context, raw q in, rotated q and out
    # written, the new token's k/v read and appended, block table, split-K partials
    # written and read back
    if T == BALANCED:
        parts = _balanced_partials(lengths, hkv, hq // hkv, sms)
    else:   # partitions of split sequences, one partial per query head each
        parts = sum(math.ceil(L / T) for L in lengths if L > T) * hq
    alg = (kv_bytes_rank + 3 * B * hq * d * 2 + 2 * 2 * B * hkv * d * 2 + sum(pages_per) * 4
           + B * 4 + 2 * parts * (d + 1) * 4)
    peaks = _peaks()
    achieved = alg / (k_ms * 1e-3) / 1e9
    res = {"value": value, "ms_per_step": ms, "tokens_per_s": B / (ms * 1e-3),
           "hbm_frac_step": value / world / peaks["hbm_gbs"],
           "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                        "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                        "traffic": _profile_traffic(name, world),
                        "kernel": ("paged_decode_tma_kernel<128,bf16,64,fused> (balanced split, "
                                   "in-kernel merge)") if T == BALANCED else
                                  "paged_decode_tma_kernel<128,bf16,64,fused> + lse_merge_kernel",
                        "kernel_ms": k_ms, "kernel_ms_how": k_how, "algorithmic_bytes": alg,
                        "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json hbm_gbs)"},
           "clocks": clocks, "e2e": e2e,
           "gpu_launches_per_step": 1 if T == BALANCED else 2}
    if tri is not None:
        res["reference_gpu_kernel"] = tri
    del graphs, sets
    torch.cuda.empty_cache()
    return res


# ---------------------------------------------------------------------------
# Config 5: full decode step with head-sharded TP
# ---------------------------------------------------------------------------
class PhaseTimer:
    """``model.mark`` hook: a timing event node after each phase of a captured step;
    ``split()`` sums the intervals per phase name after a replay."""

    def __init__(self):
        self.events, self.labels = [], []

    def __call__(self, label: str) -> None:
        if not torch.cuda.is_current_stream_capturing():
            return
        e = torch.cuda.Event(enable_timing=True, external=True)
        e.record()
        self.events.append(e)
        self.labels.append(label)

    def split(self) -> tuple[dict, float]:
        out: dict = {}
        for i in range(1, len(self.events)):
            dt = self.events[i - 1].elapsed_time(self.events[i])
            out[self.labels[i]] = out.get(self.labels[i], 0.0) + dt
        total = self.events[0].elapsed_time(self.events[-1]) if len(self.events) > 1 else 0.0
        return out, total


def _agree(ok: bool, world: int) -> bool:
    """True when every rank reports ok (a collective: call it on every rank)."""
    if world == 1:
        return ok
    import torch.distributed as dist

    t = torch.tensor([1 if ok else 0], dtype=torch.int32, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


def _status_word(model, cache) -> int:
    """OR of the step's device status words (attention and fused all-reduce); read
    without raising, then cleared."""
    torch.cuda.synchronize()
    words = [cache.layer_caches[0].status]
    if model.tp.fused is not None:
        words.append(model.tp.fused.status)
    w = 0
    for t in words:
        w |= int(t.item())
        t.zero_()
    return w


def measure_c5(world: int, rank: int, dev, steps: int = 128, warmup: int = 5,
               parity_steps: int = 8, variants=("fused", "nccl"), tc_gemms=None,
               with_e2e: bool = True) -> dict:
    """Config 5 at TP = world: tokens/s of the whole-step CUDA graph (32 layers + lm_head
    + argmax) for each all-reduce variant, the per-phase split of one step, and at
    TP > 1 the logits against a TP1 model of the same weights on rank 0."""
    from llm_cuda_b200.kernels.decode_attention import BALANCED
    from llm_cuda_b200.models.llama3.decode_model import (
        DecodeConfig, DecodeGraph, Llama3DecodeModel, TensorParallel)

    cfg = DecodeConfig()
    B, prompt, P = 64, 2048, 16
    cap = prompt + steps + parity_steps + 16
    tp = TensorParallel(rank, world)
    model = Llama3DecodeModel.random_init(cfg, dev, torch.bfloat16, seed=1005, tp=tp,
                                          max_positions=cap)
    if tc_gemms is not None:
        model.tc_projections = set(x for x in tc_gemms.split(",") if x)
    if world > 1:
        model.enable_fused_allreduce(rows_cap=B)   # one-shot NVLink AR + add + RMSNorm
    fused_ar = model.tp.fused
    cache = model.make_cache(B, cap, page_size=P, shuffle_seed=1005 + rank)
    ids = torch.randint(0, cfg.vocab_size, (B, prompt),
                        generator=torch.Generator().manual_seed(1005)).to(dev)
    with torch.no_grad():
        prefill_logits = model.prefill(ids, cache)
    first = prefill_logits.argmax(-1)
    torch.cuda.synchronize()
    lens0 = cache.get_layer(0).seq_lens.clone()
    w_bytes, _ = model.bytes_per_step(cache)
    kv_total = sum((prompt + i + 1) * B * model.hkv * cfg.head_dim * 2 * 2 * cfg.num_hidden_layers
                   for i in range(steps))
    peaks = _peaks()
    bytes_rank = w_bytes + kv_total / steps
    out = {"config": {"workload": "config5 Llama-3-8B-shaped decode: 32 layers, hidden 4096, "
                                  "Hq32 Hkv8 d128, ffn 14336, vocab 128256, B64, KV prefilled "
                                  "to 2048 (page 16), greedy decode",
                      "tp": world, "steps": steps,
                      "graph": "whole step (32 layers + lm_head + argmax) replayed from one "
                               "CUDA graph",
                      "weight_bytes_per_rank": w_bytes,
                      "kv_bytes_per_rank_per_step_avg": kv_total / steps}}

    def reset(graph):
        for lc in cache.layer_caches:
            lc.seq_lens.copy_(lens0)
            lc.host_lengths = [prompt] * B
        graph.ids.copy_(first)

    record = None
    clocks = []
    for vi, variant in enumerate(variants if world > 1 else ("fused",)):
        model.tp.fused = fused_ar if variant == "fused" else None
        graph = DecodeGraph(model, cache, first, partition_tokens=BALANCED)
        if vi == 0 and world > 1 and parity_steps:
            # logits and ids of the first steps, for the TP1 comparison on rank 0
            record = {"ids": [], "logits": []}
            reset(graph)
            for _ in range(parity_steps):
                record["ids"].append(graph.ids.clone())
                graph.replay()
                record["logits"].append(graph.logits.float().clone())
            torch.cuda.synchronize()
        reset(graph)
        for _ in range(max(3, warmup)):
            graph.replay()
        reset(graph)
        word = _status_word(model, cache)
        if not _agree(word == 0, world):
            # Every rank leaves this variant together (a device wait timed out on some
            # rank); the status word is reported, the next variant runs without it.
            out[variant] = {"error": f"device status {word:#x} on rank {rank} in warm-up"}
            record = None
            del graph
            torch.cuda.synchronize()
            if variant == "fused":
                fused_ar = None
            continue
        _barrier(world)
        clock = ClockSampler(dev.index if world > 1 else 0)
        with clock:
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            _barrier(world)
            torch.cuda.synchronize()
            stream = torch.cuda.current_stream(dev)
            torch.cuda.nvtx.range_push(f"c5_steps_{variant}")
            e0.record(stream)
            for _ in range(steps):
                graph.replay()
            e1.record(stream)
            torch.cuda.nvtx.range_pop()
            torch.cuda.synchronize()
            _barrier(world)
        clocks.append(clock.summary())
        word = _status_word(model, cache)
        ms = _max_over_ranks(e0.elapsed_time(e1) / steps, world)
        if not _agree(word == 0, world):
            out[variant] = {"error": f"device status {word:#x} on rank {rank} while timed"}
            if variant == "fused":
                fused_ar, record = None, None
        else:
            out[variant] = {"tokens_per_s": B / (ms * 1e-3), "ms_per_step": ms,
                            "hbm_gbs_per_gpu": bytes_rank / (ms * 1e-3) / 1e9,
                            "hbm_frac_per_gpu": bytes_rank / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"]}
        # The step graph may hold captured NCCL all-reduces: release it before the next.
        del graph
        torch.cuda.synchronize()
    good = [v for v in ("fused", "nccl") if "tokens_per_s" in out.get(v, {})]
    if not good:
        raise RuntimeError(f"config 5: no variant completed: {out}")
    main_v = "fused" if "fused" in good else good[0]
    out["tokens_per_s"] = out[main_v]["tokens_per_s"]
    out["ms_per_step"] = out[main_v]["ms_per_step"]
    out["hbm_frac_per_gpu"] = out[main_v]["hbm_frac_per_gpu"]
    out["reported_variant"] = main_v
    out["faster_allreduce"] = (max(good, key=lambda v: out[v]["tokens_per_s"]) if world > 1
                               else "none (TP1)")
    out["roofline_ms_per_step"] = bytes_rank / (peaks["hbm_gbs"] * 1e9) * 1e3

    # ---- per-phase split of one step (the reported variant): timing event nodes
    # between the phases of an instrumented copy of the graph ----
    model.tp.fused = fused_ar
    timer = PhaseTimer()
    model.mark = timer
    try:
        graph = DecodeGraph(model, cache, first, partition_tokens=BALANCED)
        model.mark = None
        reset(graph)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        split, total = timer.split()
        split_max = {k: _max_over_ranks(v, world) for k, v in sorted(split.items())}
        total = _max_over_ranks(total, world)
        out["split_ms"] = {k: round(v, 4) for k, v in split_max.items()}
        out["split_total_ms"] = total
        out["split_how"] = ("one replay of an instrumented step graph with a timing event "
                            "node after every phase of every layer (the nodes stop launch "
                            "overlap, so the total exceeds ms_per_step); max over ranks")
        del graph
    except Exception as ex:
        out["split_ms"] = {"unavailable": f"{type(ex).__name__}: {str(ex)[:160]}"}
    finally:
        model.mark = None
    word = _status_word(model, cache)
    if not _agree(word == 0, world):
        out["split_ms"] = {"unavailable": f"device status {word:#x} on rank {rank}"}

    # ---- e2e: host ids in (pinned), greedy ids out, eager public API per step ----
    if with_e2e:
        for lc in cache.layer_caches:
            lc.seq_lens.copy_(lens0)
            lc.host_lengths = [prompt] * B
        h_ids = torch.empty(B, dtype=torch.long, pin_memory=True)
        h_ids.copy_(first.cpu())
        h_out = torch.empty(B, dtype=torch.long, pin_memory=True)
        e2e_steps = min(steps, 16)
        _barrier(world)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        with torch.no_grad():
            for _ in range(e2e_steps):
                d_ids = h_ids.to(dev, non_blocking=True)
                nxt = model.decode_step(d_ids, cache, partition_tokens=BALANCED).argmax(-1)
                h_out.copy_(nxt, non_blocking=True)
                torch.cuda.synchronize()
                h_ids.copy_(h_out)
        e2e_ms = _max_over_ranks((time.perf_counter() - t0) / e2e_steps * 1e3, world)
        out["e2e"] = {"value": B / (e2e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                      "h2d_bytes_per_step": B * 8, "d2h_bytes_per_step": B * 8,
                      "path": "Llama3DecodeModel.decode_step eager + argmax, host ids in/out"}
        word = _status_word(model, cache)
        if not _agree(word == 0, world):
            out["e2e"] = {"error": f"device status {word:#x} on rank {rank}"}

    # ---- TP=N against TP1 (rank 0): same weights, same prompt, teacher-forced ids ----
    if record is not None:
        _barrier(world)
        if rank == 0:
            del cache
            torch.cuda.empty_cache()
            ref = Llama3DecodeModel.random_init(cfg, dev, torch.bfloat16, seed=1005,
                                                tp=TensorParallel(0, 1), max_positions=cap)
            rc = ref.make_cache(B, cap, page_size=P, shuffle_seed=1005)
            with torch.no_grad():
                pl1 = ref.prefill(ids, rc)
                diffs, agree = [], []
                for t in range(parity_steps):
                    lg = ref.decode_step(record["ids"][t], rc, partition_tokens=BALANCED).float()
                    ln = record["logits"][t]
                    diffs.append((lg - ln).abs().max().item())
                    agree.append((lg.argmax(-1) == ln.argmax(-1)).float().mean().item())
            rc.check_status()
            out["parity_vs_tp1"] = {
                "steps": parity_steps,
                "prefill_logits_max_abs_diff": (pl1.float() - prefill_logits.float()).abs().max().item(),
                "logits_max_abs_diff": max(diffs), "logits_max_abs_diff_per_step": diffs,
                "logits_max_abs": max(r.abs().max().item() for r in record["logits"]),
                "greedy_agreement": statistics.mean(agree),
                "how": "rank 0 runs a TP1 model of the same seeded weights and prompt; each "
                       "step is fed the TP=N run's input ids (teacher forcing)"}
            del ref, rc
            torch.cuda.empty_cache()
        _barrier(world)
    out["clocks"] = _merge_clocks(clocks)
    out["gpu_launches_per_step"] = _c5_launches(cfg, world)
    if fused_ar is not None:
        _barrier(world)
        fused_ar.close()
    return out


def _c5_launches(cfg, world: int) -> int:
    """This package's kernels per config-5 step: per layer the fused attention launch,
    add/RMSNorm (or the fused all-reduce) twice and SwiGLU; then the final norm,
    lm_head (tcgen05 GEMM) and argmax.  The layer projections are cuBLAS unless set."""
    return cfg.num_hidden_layers * 4 + 3


def run_c5_main(args):
    """--workload c5: config 5 alone, its own JSON line (tokens/s)."""
    from llm_cuda_b200 import _native as N

    N.load()
    world, rank, local = _dist_setup()
    dev = torch.device("cuda", local if world > 1 else 0)
    r = measure_c5(world, rank, dev, steps=args.steps, warmup=args.warmup,
                   tc_gemms=args.tc_gemms,
                   variants=("nccl", "fused") if args.nccl_allreduce else ("fused", "nccl"))
    if rank == 0:
        main_v = r["reported_variant"]
        if args.nccl_allreduce and world > 1 and "tokens_per_s" in r.get("nccl", {}):
            main_v = "nccl"
        line = {
            "metric": "decode tokens/s (config 5 full decode step)",
            "value": r[main_v]["tokens_per_s"], "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": r[main_v]["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init N(0,0.02) weights, random prompt ids)",
            "config": dict(r["config"], parallelism=f"tp{world} (head-sharded)"),
            "c5": r, "e2e": r.get("e2e"),
            "gpu_launches": r["gpu_launches_per_step"] * args.steps, "clocks": r["clocks"],
        }
        print(json.dumps(line), flush=True)
    _finish(world)


def _finish(world):
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        sys.stdout.flush()
        os._exit(0)   # graphs holding captured NCCL work must not block the teardown


def run_main(args):
    from llm_cuda_b200 import _native as N

    N.load()
    world, rank, local = _dist_setup()
    dev = torch.device("cuda", local if world > 1 else 0)
    name = args.workload
    w, lengths = _workload(name, args.scaling, world)
    extras = not args.no_extras
    main = measure_decode(name, w, lengths, args.steps, args.warmup, world, rank, dev,
                          with_e2e=True, with_triton=extras and world == 1)
    subs = {}
    if extras and world == 1 and name == "c2":
        for sub in ("c3", "c4"):
            ws, ls = _workload(sub, "weak", 1)
            try:
                r = measure_decode(sub, ws, ls, min(args.steps, 100), 3, world, rank, dev,
                                   with_e2e=False)
                subs[sub] = {"workload": ws["desc"], "value": r["value"], "unit": "GB/s",
                             "ms_per_step": r["ms_per_step"],
                             "tokens_per_s": r["tokens_per_s"],
                             "roofline_frac": r["roofline"]["frac"],
                             "kernel_ms": r["roofline"]["kernel_ms"],
                             "algorithmic_bytes": r["roofline"]["algorithmic_bytes"],
                             "clocks": r["clocks"]}
            except Exception as ex:
                subs[sub] = {"unavailable": f"{type(ex).__name__}: {str(ex)[:200]}"}
    c5 = None
    if extras and name == "c2":
        # A Python error raised on every rank alike is reported and the line still
        # printed; device errors are agreed on inside measure_c5.
        try:
            c5 = measure_c5(world, rank, dev, steps=128, warmup=5)
        except Exception as ex:
            import traceback

            traceback.print_exc()
            c5 = {"unavailable": f"{type(ex).__name__}: {str(ex)[:200]}"}
    if rank == 0:
        cpu = None
        if world == 1 and args.cpu_budget > 0:
            try:
                cpu = reference_cpu_baseline(w, lengths, args.cpu_budget)
            except Exception as ex:
                cpu = {"unavailable": f"{type(ex).__name__}: {str(ex)[:200]}"}
            try:
                cpu["port"] = port_cpu_baseline(w, lengths, min(5.0, args.cpu_budget))
            except Exception as ex:
                cpu["port"] = {"unavailable": f"{type(ex).__name__}: {str(ex)[:200]}"}
        clocks = _merge_clocks([main["clocks"]] + [s.get("clocks") for s in subs.values()]
                               + ([c5["clocks"]] if c5 and "clocks" in c5 else []))
        launches = main["gpu_launches_per_step"] * args.steps
        line = {
            "metric": "decode-attn KV GB/s", "value": main["value"], "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": main["ms_per_step"], "higher_is_better": True,
            "scaling": w["scaling"], "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) K/V pages, q/k/v of the new token)",
            "tokens_per_s": main["tokens_per_s"], "hbm_frac_step": main["hbm_frac_step"],
            "config": _config(w, lengths, world),
            "roofline": main["roofline"], "cpu_baseline": cpu, "e2e": main["e2e"],
            "gpu_launches": launches,
            "gpu_launches_note": "timed region only (the decode-attention steps); the c5 "
                                 "key gives its own per-step count",
            "clocks": clocks,
        }
        if "reference_gpu_kernel" in main:
            line["reference_gpu_kernel"] = main["reference_gpu_kernel"]
        line.update(subs)
        if c5 is not None:
            line["c5"] = c5
            if "tokens_per_s" in c5:
                line["c5_tokens_per_s"] = c5["tokens_per_s"]
                line["c5_ms_per_step"] = c5["ms_per_step"]
                line["c5_hbm_frac_per_gpu"] = c5["hbm_frac_per_gpu"]
        print(json.dumps(line), flush=True)
    _finish(world)


def run_gemm(args):
    """--gemm N,K: the tcgen05 decode GEMM y[64, N] = x[64, K] W[N, K]^T alone, on W
    copies rotating over >= 300 MB (no launch finds its weights in L2); one JSON line
    with the weight-streaming rate and cuBLAS on the same shape."""
    from llm_cuda_b200 import _native as N
    from llm_cuda_b200.kernels.step_ops import decode_gemm

    N.load()
    n_out, k = (int(v) for v in args.gemm.split(","))
    mb = args.gemm_rows
    dev = torch.device("cuda", 0)
    nw = max(2, -(-300_000_000 // (n_out * k * 2)))
    g = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(mb, k, device=dev, generator=g).bfloat16()
    ws = [(0.02 * torch.randn(n_out, k, device=dev, generator=g)).bfloat16() for _ in range(nw)]
    for i in range(max(3, args.warmup)):
        y = decode_gemm(x, ws[i % nw])
    torch.cuda.synchronize()
    err = (y.float() - x.float() @ ws[(max(3, args.warmup) - 1) % nw].float().T).abs().max().item()
    res = {}
    for label, fn in (("tcgen05", lambda i: decode_gemm(x, ws[i % nw])),
                      ("cublas", lambda i: torch.nn.functional.linear(x, ws[i % nw]))):
        for i in range(3):
            fn(i)
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(gr, stream=s):
                for i in range(nw * max(1, 20 // nw)):
                    fn(i)
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize()
        per = nw * max(1, 20 // nw)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = max(1, args.steps // per)
        e0.record()
        for _ in range(reps):
            gr.replay()
        e1.record()
        torch.cuda.synchronize()
        res[label] = e0.elapsed_time(e1) / (reps * per) * 1e3
    print(json.dumps({"metric": "decode GEMM weight GB/s",
                      "value": n_out * k * 2 / res["tcgen05"] / 1e3, "unit": "GB/s",
                      "us_per_call": res["tcgen05"], "cublas_us_per_call": res["cublas"],
                      "config": {"N": n_out, "K": k, "Mb": mb, "weight_copies": nw,
                                 "timing": "CUDA graph of back-to-back calls"},
                      "max_abs_err_vs_fp32": err}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + ["c5"], default="c2")
    ap.add_argument("--no-extras", action="store_true",
                    help="only the selected workload (no c3/c4/c5 sub-results, no reference "
                         "GPU kernel, no CPU baseline)")
    ap.add_argument("--cpu-budget", type=float, default=15.0,
                    help="seconds of reference CPU-path sampling at N=1 (0: skip)")
    ap.add_argument("--tc-gemms", default=None,
                    help="config 5: comma list of decode projections (qkv,o,gate_up,down) on "
                         "the tcgen05 GEMM instead of cuBLAS (default: the model's choice)")
    ap.add_argument("--nccl-allreduce", action="store_true",
                    help="config 5 at N>1: report the NCCL all-reduce variant as the value")
    ap.add_argument("--scaling", choices=["weak", "strong"], default="weak",
                    help="N>1: weak = N x the config's batch, head-sharded (per-GPU work "
                         "fixed); strong = the config's batch split over N GPUs")
    ap.add_argument("--gemm", default=None, metavar="N,K",
                    help="time the tcgen05 decode GEMM alone (profiling aid)")
    ap.add_argument("--gemm-rows", type=int, default=64)
    args = ap.parse_args()
    if args.gemm:
        run_gemm(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.workload == "c5":
        if args.impl == "reference":
            if int(os.environ.get("RANK", "0")) == 0:
                print(json.dumps({"impl": "reference", "unavailable": "config 5 reference arm "
                                  "not run: the CPU model at Llama-3-8B size takes minutes per "
                                  "step"}))
            return
        run_c5_main(args)
        return
    w, lengths = _workload(args.workload, args.scaling, world)
    if args.impl == "reference":
        run_reference(args, args.workload, w, lengths, _config(w, lengths, world))
    else:
        run_main(args)


if __name__ == "__main__":
    main()
