"""Fused NVLink all-reduce + residual add + RMSNorm on 2 and 4 GPUs (skipped with fewer),
both algorithms (one-shot and two-shot).

Each rank runs in its own process on its own GPU (NCCL process group for the handle
exchange and for the reference all-gather).  Checked against an fp32 reference built
from all ranks' partials: x bit-exact (same fp32 sum in rank order, same roundings),
h within the bf16 bar; both ranks hold identical results; eager calls across both
buffer parities and a CUDA graph replayed several times; and the TP2 decode model's
steps with the fused kernel against the same steps with NCCL.
"""

import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

ROWS, HIDDEN = 64, 4096


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _reference(partials, x, w, eps):
    s = torch.zeros_like(partials[0], dtype=torch.float32)
    for p in partials:            # rank order, fp32
        s += p.float()
    xn = (x.float() + s.to(x.dtype).float()).to(x.dtype)
    xf = xn.float()
    h = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()
    return xn, h


def _worker(rank, world, port, q, algo):
    import torch.distributed as dist

    os.environ["LLMC_AR_ALGO"] = algo      # read once, at the first call in this process

    from llm_cuda_b200.kernels.allreduce import NvlinkAllReduce

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    out = {}
    try:
        ar = NvlinkAllReduce(None, rank, world, ROWS, HIDDEN, torch.bfloat16, dev)
        w = (1 + 0.1 * torch.randn(HIDDEN, generator=torch.Generator().manual_seed(1))).bfloat16().to(dev)
        errs = []
        for it in range(5):                       # both buffer parities, several epochs
            g = torch.Generator().manual_seed(100 * it + rank)
            part = torch.randn(ROWS, HIDDEN, generator=g).bfloat16().to(dev)
            x0 = torch.randn(ROWS, HIDDEN, generator=torch.Generator().manual_seed(7 + it)).bfloat16().to(dev)
            x = x0.clone()
            h = ar.add_rmsnorm(part, x, w, 1e-5)
            torch.cuda.synchronize()
            ar.check_status()
            parts = [torch.empty_like(part) for _ in range(world)]
            dist.all_gather(parts, part)
            xr, hr = _reference(parts, x0, w, 1e-5)
            errs.append((torch.equal(x, xr), (h.float() - hr).abs().max().item()))
            xs = [torch.empty_like(x) for _ in range(world)]
            dist.all_gather(xs, x)
            hs = [torch.empty_like(h) for _ in range(world)]
            dist.all_gather(hs, h)
            errs.append((all(torch.equal(xs[0], t) for t in xs) and
                         all(torch.equal(hs[0], t) for t in hs), 0.0))
        # a CUDA graph of three calls, replayed three times
        part = torch.randn(ROWS, HIDDEN, generator=torch.Generator().manual_seed(55 + rank)).bfloat16().to(dev)
        x = torch.zeros(ROWS, HIDDEN, dtype=torch.bfloat16, device=dev)
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(graph, stream=s):
                for _ in range(3):
                    hg = ar.add_rmsnorm(part, x, w, 1e-5)
        torch.cuda.current_stream(dev).wait_stream(s)
        dist.barrier()
        x.zero_()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        ar.check_status()
        parts = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(parts, part)
        xr = torch.zeros_like(x)
        for _ in range(9):
            xr, hr = _reference(parts, xr, w, 1e-5)
        errs.append((torch.equal(x, xr), (hg.float() - hr).abs().max().item()))
        out["kernel"] = errs
        del graph
        dist.barrier()
        ar.close()

        # TP decode model: fused NVLink path vs NCCL path, same weights and tokens
        from llm_cuda_b200.models.llama3.decode_model import (
            DecodeConfig, Llama3DecodeModel, TensorParallel)

        cfg = DecodeConfig(vocab_size=1024, hidden_size=1024, intermediate_size=2048,
                           num_hidden_layers=2, num_attention_heads=16, num_key_value_heads=8)
        # Greedy ids of the NCCL run are fed to both runs (teacher forcing): a last-bit
        # difference that flips one argmax would otherwise make every later step of the
        # two runs decode different tokens.
        logits, fed = [], []
        for fused in (False, True):
            m = Llama3DecodeModel.random_init(cfg, dev, torch.bfloat16, seed=3,
                                              tp=TensorParallel(rank, world), max_positions=256)
            if fused:
                m.enable_fused_allreduce(rows_cap=8)
            cache = m.make_cache(8, 256, 16, shuffle_seed=1)
            ids = torch.randint(0, cfg.vocab_size, (8, 20), generator=torch.Generator().manual_seed(9)).to(dev)
            with torch.no_grad():
                nxt = m.prefill(ids, cache).argmax(-1)
                steps = []
                for t in range(4):
                    if fused:
                        nxt = fed[t]
                    else:
                        fed.append(nxt.clone())
                    lg = m.decode_step(nxt, cache)
                    steps.append(lg.float().cpu())
                    nxt = lg.argmax(-1)
            torch.cuda.synchronize()
            if fused:
                m.tp.fused.check_status()
                dist.barrier()
                m.tp.fused.close()
            logits.append(torch.stack(steps))
        scale = logits[0].abs().max().item()
        out["model"] = ((logits[0] - logits[1]).abs().max().item(), scale)
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,algo", [(2, "one_shot"), (2, "two_shot"), (4, "one_shot"),
                                        (4, "two_shot")])
def test_fused_allreduce_add_rmsnorm(world, algo):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, algo)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank in range(world):
        for exact, err in res[rank]["kernel"]:
            assert exact
            assert err <= 2e-2
        err, scale = res[rank]["model"]
        assert err <= 0.05 * scale + 2e-2, (err, scale)
