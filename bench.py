"""Decode-attention benchmark (driver contract: one JSON line from rank 0).

A step is one pass of the hot path over one batch: fused RoPE + KV-page append of
the new token of every sequence, paged GQA flash-decode over the whole context,
and the split-K log-sum-exp merge.  Default workload = BASELINE config 2
(Llama-3-8B decode attention: B64 Hq32 Hkv8 d128, context 4096, page 16,
shuffled block tables, bf16).  Under torchrun with N ranks the step is
KV-head sharded (each rank owns Hkv/N KV heads and their query heads, as the
reference's column split of q/k/v_proj) — strong scaling, no data-path
collective.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c2|c3|c4|c5] [--compare-triton]

``--impl reference`` times the reference's CPU path (the oracle restatement in
``oracle/``) on the host cores with the same metric; under torchrun only rank 0
runs it.
"""

from __future__ import annotations

import argparse
import json
import math
import os
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

WORKLOADS = {
    # name: (B, Hq, Hkv, d, lengths-spec, page, scale, partition, seed, description)
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


# ---------------------------------------------------------------------------
# CPU baseline: the oracle restatement of the reference's CPU decode path
# ---------------------------------------------------------------------------
def _cpu_unit(rng, L, G, d, dt):
    """One (sequence, KV head) unit of a decode step for the oracle."""
    from oracle import decode_oracle as O

    q = O.round_to(rng.standard_normal((G, d), dtype=np.float32), dt)
    k = O.round_to(rng.standard_normal((1, L, d), dtype=np.float32), dt)
    v = O.round_to(rng.standard_normal((1, L, d), dtype=np.float32), dt)
    cos, sin = O.build_rope_cache([L - 1], d, THETA, dt)
    return q, k, v, cos, sin


def _run_cpu_unit(u, dt):
    from oracle import decode_oracle as O

    q, k, v, cos, sin = u
    qr = O.apply_rotary(q[:, None], cos, sin, dt)[:, 0]
    return O.decode_attention(qr, k, v, dt)


def cpu_baseline(w: dict, lengths, budget_s: float) -> dict:
    """Time the oracle on (sequence, KV head) units of the workload for ~budget_s."""
    dt = "bf16"
    G, d = w["Hq"] // w["Hkv"], w["d"]
    rng = np.random.default_rng(0)
    L = int(lengths[len(lengths) // 2])
    u = _cpu_unit(rng, L, G, d, dt)
    _run_cpu_unit(u, dt)  # warm
    n, kv_bytes = 0, 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        _run_cpu_unit(u, dt)
        n += 1
        kv_bytes += L * d * 2 * 2
    el = time.perf_counter() - t0
    return {"value": kv_bytes / el / 1e9, "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{n} (sequence, KV head) units of ctx {L}, G={G}, d={d}, bf16 rounding "
                      f"emulated, {el:.1f} s; numpy/OpenBLAS with {os.cpu_count()} threads"}


def run_reference(args, w, lengths):
    """--impl reference: the reference's CPU path (oracle port) on this host's cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    dt = "bf16"
    G, d = w["Hq"] // w["Hkv"], w["d"]
    rng = np.random.default_rng(0)
    L = int(lengths[len(lengths) // 2])
    u = _cpu_unit(rng, L, G, d, dt)
    t0 = time.perf_counter()
    _run_cpu_unit(u, dt)
    t_unit = max(time.perf_counter() - t0, 1e-4)
    budget = 150.0 / max(1, args.steps + args.warmup)
    units = max(1, int(budget / t_unit))
    for _ in range(args.warmup):
        for _ in range(units):
            _run_cpu_unit(u, dt)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for _ in range(units):
            _run_cpu_unit(u, dt)
    el = time.perf_counter() - t0
    kv = units * args.steps * L * d * 2 * 2
    value = kv / el / 1e9
    full_kv = sum(lengths) * w["Hkv"] * d * 2 * 2
    line = {
        "impl": "reference", "metric": "decode-attn KV GB/s", "value": value, "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3 * (full_kv / (units * L * d * 4)),
        "higher_is_better": True, "scaling": w["scaling"], "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": {"workload": w["desc"], "sample_units_per_step": units},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": f"{units} (sequence, KV head) units of ctx {L} per step "
                                   "(oracle restatement of attention.py:56-89 + rotary.py:104-109)"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def _dist_setup(args):
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


def triton_reference_compare(sets, lengths) -> dict:
    """Time the reference's own GPU kernel, ``triton_decode_attention``
    (``src/llm_cuda/kernels/triton/decode_attention.py:204-287`` of llm-cuda,
    installed unmodified in ``baseline/_ref``), on this step's data.  It needs dense
    ``[B, Hkv, L, d]`` K/V, so the pages are gathered first (the reference's
    ``get_kv``, ``kv_cache.py:65-83``, does the same copy each step); the gather is
    timed separately."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "llm_cuda")):
        return {"unavailable": "baseline/_ref not installed"}
    if len(set(lengths)) != 1:
        return {"unavailable": "ragged batch: the reference kernel takes one kv_len"}
    # The unmodified reference kernel reads a module-level float inside @triton.jit,
    # which Triton 3.6 rejects unless this documented Triton switch is set.
    os.environ.setdefault("TRITON_ALLOW_NON_CONSTEXPR_GLOBALS", "1")
    sys.path.insert(0, ref)
    from llm_cuda.kernels.triton.decode_attention import triton_decode_attention as ref_decode

    st = sets[0]
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
            segs = owner(x0 + c - 1) - owner(x0) + 1
            if segs > 1:
                n += segs * h
        x0 += c
    return n


def run_ours(args, name, w, lengths):
    from llm_cuda_b200 import _native as N
    from llm_cuda_b200.kernels.decode_attention import (
        BALANCED, paged_decode, rope_append_decode)
    from llm_cuda_b200.models.llama3 import PagedKVLayerCache, RopeTable, make_block_table
    from llm_cuda_b200.models.llama3.kv_cache import GraphedDecodeStep

    N.load()
    world, rank, local = _dist_setup(args)
    dev = torch.device("cuda", local if world > 1 else 0)
    B, Hq, Hkv, d, P = w["B"], w["Hq"], w["Hkv"], w["d"], w["P"]
    if Hkv % world:
        raise SystemExit(f"KV heads {Hkv} do not shard over {world} ranks")
    hkv, hq = Hkv // world, Hq // world              # this rank's heads (TP shard)
    dtype = torch.bfloat16
    pages_per = [math.ceil(L / P) for L in lengths]
    max_pages = max(pages_per)
    kv_bytes_rank = sum(lengths) * hkv * d * 2 * 2    # K and V read per step
    n_sets = max(1, math.ceil(3 * L2_BYTES / kv_bytes_rank)) if kv_bytes_rank < 3 * L2_BYTES else 1
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
        # attention; the merge launch combines split-K partials and advances seq_lens.
        c = st["cache"]
        c.seq_lens.copy_(st["base"])          # every step attends exactly the configured context
        c.host_lengths = list(base_host)
        rope_append_decode(st["q"], st["k"], st["v"], c.key_pages, c.value_pages,
                           c.block_table, c.seq_lens, rope.cos, rope.sin, host_lens=base_host,
                           partition_tokens=T, out=st["out"], q_out=st["q_rot"],
                           workspace=c.workspace, status=c.status, events=ev)

    # eager warm-up (also allocates the split-K workspace before capture)
    for st in sets:
        step(st)
    torch.cuda.synchronize()
    for st in sets:
        st["cache"].check_status()

    # one CUDA graph per input set
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    graphs = []
    with torch.cuda.stream(stream):
        for st in sets:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                step(st)
            graphs.append(g)
    torch.cuda.current_stream(dev).wait_stream(stream)
    torch.cuda.synchronize()

    with torch.cuda.stream(stream):
        for i in range(max(3, args.warmup)):
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
            for i in range(args.steps):
                graphs[i % n_sets].replay()
            e1.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        _barrier(world)
        ms = e0.elapsed_time(e1) / args.steps
        # ---- decode-kernel duration on its launching stream (eager launches) ----
        kreps = min(args.steps, 200)
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(kreps)]
        with torch.cuda.stream(stream):
            for i in range(kreps):
                # A short device sleep ahead of each step keeps the GPU busy while the
                # host issues the bracketed launches, so the events time device work only.
                torch.cuda._sleep(200_000)
                step(sets[i % n_sets], evs[i])
        torch.cuda.synchronize()
        k_ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
    clocks = clock.summary()
    for st in sets:
        st["cache"].check_status()
    tri = None
    if args.compare_triton:
        try:
            tri = triton_reference_compare(sets, lengths)
        except Exception as e:  # informative only; never fails the bench line
            tri = {"unavailable": f"{type(e).__name__}: {str(e)[:200]}"}
    ms = _max_over_ranks(ms, world)
    k_ms = _max_over_ranks(k_ms, world)

    # ---- e2e through the public API with host buffers ----
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
    # The public graphed step (GraphedDecodeStep) of each input buffer: one graph
    # launch per step, reading that buffer and writing its own output buffer.
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
    e2e_steps = max(10, min(args.steps, 500))
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

    total_kv = sum(lengths) * Hkv * d * 2 * 2         # all ranks together
    value = total_kv / (ms * 1e-3) / 1e9
    tokens_s = B / (ms * 1e-3)
    # algorithmic bytes of the fused decode launch + its merge launch on one rank: K/V
    # of the whole context, raw q in, rotated q and out written, the new token's k/v
    # read and appended, block table, split-K partials written and read back
    if T == BALANCED:
        parts = _balanced_partials(lengths, hkv, hq // hkv, sms)
    else:   # partitions of split sequences, one partial per query head each
        parts = sum(math.ceil(L / T) for L in lengths if L > T) * hq
    alg = (kv_bytes_rank + 3 * B * hq * d * 2 + 2 * 2 * B * hkv * d * 2 + sum(pages_per) * 4
           + B * 4 + 2 * parts * (d + 1) * 4)
    achieved = alg / (k_ms * 1e-3) / 1e9
    peaks = _peaks()
    if rank == 0:
        cpu = cpu_baseline(w, lengths, args.cpu_budget) if world == 1 and args.cpu_budget > 0 else None
        line = {
            "metric": "decode-attn KV GB/s", "value": value, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": w["scaling"], "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded N(0,1) K/V pages, q/k/v of the new token)",
            "tokens_per_s": tokens_s,
            "hbm_frac_step": value / world / peaks["hbm_gbs"],
            "config": {"workload": w["desc"], "B": B, "global_batch": B, "Hq": Hq, "Hkv": Hkv,
                       "head_dim": d,
                       "page_size": P, "context_tokens_total": sum(lengths),
                       "partition_tokens": T if T else "balanced",
                       "parallelism": f"tp{world} (KV-head sharded)",
                       "input_sets": n_sets,
                       "l2": f"KV per rank {kv_bytes_rank / 1e6:.0f} MB x {n_sets} rotating sets "
                             f"> L2 126 MB (no flush needed)",
                       "graph": "each step replayed from a CUDA graph"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                         "traffic": _profile_traffic(name, world),
                         "kernel": ("paged_decode_tma_kernel<128,bf16,64,fused> (balanced split, "
                                    "in-kernel merge)") if T == BALANCED else
                                   "paged_decode_tma_kernel<128,bf16,64,fused> + lse_merge_kernel",
                         "kernel_ms": k_ms, "algorithmic_bytes": alg,
                         "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json hbm_gbs)"},
            "cpu_baseline": cpu,
            "e2e": {"value": total_kv / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
                    "ms_per_step": e2e_ms, "tokens_per_s": B / (e2e_ms * 1e-3),
                    "h2d_bytes_per_step": h_in.numel() * h_in.element_size(),
                    "d2h_bytes_per_step": h_out[0].numel() * h_out[0].element_size(),
                    "path": "GraphedDecodeStep (the fused RoPE+append+decode step, one graph "
                            "launch per step) with pinned host in/out, copies on a second "
                            "stream overlapping compute"},
            # per step: the fused decode launch (+ the merge launch with uniform
            # partitions); the length reset is a graph memcpy node, not a kernel
            "gpu_launches": (1 if T == BALANCED else 2) * args.steps,
            "clocks": clocks,
        }
        if tri is not None:
            line["reference_gpu_kernel"] = tri
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def run_c5(args):
    """Config 5: full decode step of a random-init Llama-3-8B-shaped model, B=64, paged KV
    prefilled to 2048 tokens (page 16), head-sharded TP over the ranks with NCCL
    all-reduce after o_proj and down_proj; K timed greedy decode steps, each replayed
    from one CUDA graph of the whole step."""
    from llm_cuda_b200 import _native as N
    from llm_cuda_b200.kernels.decode_attention import BALANCED
    from llm_cuda_b200.models.llama3.decode_model import (
        DecodeConfig, DecodeGraph, Llama3DecodeModel, TensorParallel)

    N.load()
    world, rank, local = _dist_setup(args)
    dev = torch.device("cuda", local if world > 1 else 0)
    cfg = DecodeConfig()
    B, prompt, P = 64, 2048, 16
    steps = args.steps
    cap = prompt + steps + 16
    model = Llama3DecodeModel.random_init(cfg, dev, torch.bfloat16, seed=1005,
                                          tp=TensorParallel(rank, world), max_positions=cap)
    if args.tc_gemms is not None:
        model.tc_projections = set(x for x in args.tc_gemms.split(",") if x)
    if world > 1 and not args.nccl_allreduce:
        model.enable_fused_allreduce(rows_cap=B)   # one-shot NVLink AR + add + RMSNorm
    cache = model.make_cache(B, cap, page_size=P, shuffle_seed=1005 + rank)
    ids = torch.randint(0, cfg.vocab_size, (B, prompt),
                        generator=torch.Generator().manual_seed(1005)).to(dev)
    with torch.no_grad():
        first = model.prefill(ids, cache).argmax(-1)
    torch.cuda.synchronize()
    T = BALANCED   # the captured step re-balances on the device as contexts grow
    graph = DecodeGraph(model, cache, first, partition_tokens=T)
    lens0 = cache.get_layer(0).seq_lens.clone()

    def reset():
        for lc in cache.layer_caches:
            lc.seq_lens.copy_(lens0)
            lc.host_lengths = [prompt] * B
        graph.ids.copy_(first)

    for _ in range(max(3, args.warmup)):
        graph.replay()
        if cache.get_layer(0).host_lengths[0] >= prompt + steps:
            reset()
    reset()
    torch.cuda.synchronize()
    cache.check_status()
    w_bytes, _ = model.bytes_per_step(cache)
    kv_total = sum((prompt + i + 1) * B * model.hkv * cfg.head_dim * 2 * 2 * cfg.num_hidden_layers
                   for i in range(steps))
    _barrier(world)
    stream = torch.cuda.current_stream(dev)
    clock = ClockSampler(dev.index if world > 1 else 0)
    with clock:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        _barrier(world)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("decode_steps")
        e0.record(stream)
        for _ in range(steps):
            graph.replay()
        e1.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        _barrier(world)
    cache.check_status()
    ms = _max_over_ranks(e0.elapsed_time(e1) / steps, world)
    # e2e: host ids in (pinned), greedy ids out, eager public API per step
    reset()
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
            nxt = model.decode_step(d_ids, cache, partition_tokens=T).argmax(-1)
            h_out.copy_(nxt, non_blocking=True)
            torch.cuda.synchronize()
            h_ids.copy_(h_out)
    e2e_ms = _max_over_ranks((time.perf_counter() - t0) / e2e_steps * 1e3, world)
    clocks = clock.summary()
    peaks = _peaks()
    bytes_rank = w_bytes + kv_total / steps                 # per rank per step
    if rank == 0:
        line = {
            "metric": "decode tokens/s (config 5 full decode step)", "value": B / (ms * 1e-3),
            "unit": "tokens/s", "n_gpus": world, "steps": steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init N(0,0.02) weights, random prompt ids)",
            "hbm_gbs_per_gpu": bytes_rank / (ms * 1e-3) / 1e9,
            "hbm_frac_per_gpu": bytes_rank / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
            "config": {"workload": "config5 Llama-3-8B-shaped decode: 32 layers, hidden 4096, "
                                   "Hq32 Hkv8 d128, ffn 14336, vocab 128256, B64, KV prefilled "
                                   "to 2048 (page 16), greedy decode",
                       "parallelism": f"tp{world} (head-sharded; " + (
                           "fused one-shot NVLink all-reduce + add + RMSNorm" if model.tp.fused
                           is not None else "NCCL all-reduce") + " after o_proj/down_proj)",
                       "partition_tokens": "balanced", "graph": "whole step (32 layers + lm_head + "
                                                       "argmax) replayed from one CUDA graph",
                       "weight_bytes_per_rank": w_bytes,
                       "kv_bytes_per_rank_per_step_avg": kv_total / steps},
            "e2e": {"value": B / (e2e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": B * 8, "d2h_bytes_per_step": B * 8,
                    "path": "Llama3DecodeModel.decode_step eager + argmax, host ids in/out"},
            "gpu_launches": 3 * cfg.num_hidden_layers * steps,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    # The step graph holds captured NCCL all-reduces: release it (and the cache)
    # before the process group, whose teardown otherwise blocks on them.
    del graph
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        sys.stdout.flush()
        os._exit(0)


def run_gemm(args):
    """--gemm N,K: the tcgen05 decode GEMM y[64, N] = x[64, K] W[N, K]^T alone, on W
    copies rotating over >= 300 MB (no launch finds its weights in L2); one JSON line
    with the weight-streaming rate.  Used for the decode-GEMM profiles."""
    from llm_cuda_b200 import _native as N
    from llm_cuda_b200.kernels.step_ops import decode_gemm

    N.load()
    n_out, k = (int(v) for v in args.gemm.split(","))
    dev = torch.device("cuda", 0)
    nw = max(2, -(-300_000_000 // (n_out * k * 2)))
    g = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(64, k, device=dev, generator=g).bfloat16()
    ws = [(0.02 * torch.randn(n_out, k, device=dev, generator=g)).bfloat16() for _ in range(nw)]
    for i in range(max(3, args.warmup)):
        y = decode_gemm(x, ws[i % nw])
    torch.cuda.synchronize()
    err = (y.float() - x.float() @ ws[(max(3, args.warmup) - 1) % nw].float().T).abs().max().item()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        decode_gemm(x, ws[i % nw])
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    print(json.dumps({"metric": "decode GEMM weight GB/s", "value": n_out * k * 2 / ms / 1e6,
                      "unit": "GB/s", "ms_per_call": ms, "steps": args.steps,
                      "config": {"N": n_out, "K": k, "Mb": 64, "weight_copies": nw},
                      "max_abs_err_vs_fp32": err}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + ["c5"], default="c2")
    ap.add_argument("--compare-triton", action="store_true",
                    help="also time the reference's Triton decode kernel (baseline/_ref)")
    ap.add_argument("--cpu-budget", type=float, default=15.0,
                    help="seconds of oracle CPU-baseline sampling at N=1 (0: skip)")
    ap.add_argument("--tc-gemms", default=None,
                    help="config 5: comma list of decode projections (qkv,o,gate_up,down) on "
                         "the tcgen05 GEMM instead of cuBLAS (default: the model's choice)")
    ap.add_argument("--nccl-allreduce", action="store_true",
                    help="config 5 at N>1: NCCL all-reduce + add/RMSNorm kernel instead of the "
                         "fused one-shot NVLink kernel")
    ap.add_argument("--scaling", choices=["weak", "strong"], default="weak",
                    help="N>1: weak = N x the config's batch, head-sharded (per-GPU work "
                         "fixed); strong = the config's batch split over N GPUs")
    ap.add_argument("--gemm", default=None, metavar="N,K",
                    help="time the tcgen05 decode GEMM alone at Mb=64 (profiling aid)")
    args = ap.parse_args()
    if args.gemm:
        run_gemm(args)
        return
    if args.workload == "c5":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "config 5 reference arm not "
                              "run: the CPU model at Llama-3-8B size takes minutes per step"}))
            return
        run_c5(args)
        return
    w = dict(WORKLOADS[args.workload])
    world = int(os.environ.get("WORLD_SIZE", "1"))
    w["scaling"] = args.scaling
    if args.scaling == "weak" and world > 1:
        # Weak scaling: the config's batch per GPU, N times the sequences in all,
        # every rank holding its 1/N of the KV heads of all of them.
        w["B"] *= world
        w["desc"] += f" (global batch {w['B']} = {world} x the config's, weak scaling)"
    lengths = _lengths(args.workload, w)
    if args.impl == "reference":
        run_reference(args, w, lengths)
    else:
        run_ours(args, args.workload, w, lengths)


if __name__ == "__main__":
    main()
