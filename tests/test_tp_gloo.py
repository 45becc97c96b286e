"""Multi-rank host logic of the TP decode step on CPU ``gloo`` ranks (world size 2 and 4).

The CUDA kernels need a GPU, so the attention core is replaced by a dense torch
restatement of the reference's decode branch (RoPE, cache concat, repeat_kv,
softmax attention).  What is tested is the tensor-parallel plumbing: weight
shards in the reference's layout, per-rank heads, and the all-reduce that
replaces the reference's in-process sum of row-parallel partials.
"""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from llm_cuda_b200.models.llama3.decode_model import (
    DecodeConfig,
    Llama3DecodeModel,
    TensorParallel,
    shard_cols,
    shard_rows,
)
from llm_cuda_b200.models.llama3.rotary import build_rope_cache

CFG = DecodeConfig(vocab_size=97, hidden_size=64, intermediate_size=96, num_hidden_layers=2,
                   num_attention_heads=8, num_key_value_heads=4)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _DenseLayer:
    def __init__(self):
        self.k = None
        self.v = None

    @property
    def length(self):
        return 0 if self.k is None else self.k.shape[2]


class _DenseCache:
    def __init__(self, n):
        self.layers = [_DenseLayer() for _ in range(n)]

    def get_layer(self, i):
        return self.layers[i]


def _dense_core(cfg):
    def core(li, q, k, v, lc):
        d = q.shape[-1]
        cos, sin = build_rope_cache(1, d, cfg.rope_theta, q.device, q.dtype, lc.length)

        def rot(x):
            h = x.shape[-1] // 2
            return x * cos + torch.cat((-x[..., h:], x[..., :h]), -1) * sin

        q, k = rot(q), rot(k)
        lc.k = k if lc.k is None else torch.cat([lc.k, k], 2)
        lc.v = v if lc.v is None else torch.cat([lc.v, v], 2)
        rep = q.shape[1] // lc.k.shape[1]
        kk = lc.k.repeat_interleave(rep, 1)
        vv = lc.v.repeat_interleave(rep, 1)
        s = q @ kk.transpose(-2, -1) / d ** 0.5
        return torch.softmax(s, -1) @ vv

    return core


def _run(model, ids):
    model.attn_core = _dense_core(model.cfg)
    cache = _DenseCache(model.cfg.num_hidden_layers)
    return torch.stack([model.decode_step(ids[:, t], cache) for t in range(ids.shape[1])], 1)


def _worker(rank, world, port, ids, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        tp = TensorParallel(rank, world)
        m = Llama3DecodeModel.random_init(CFG, "cpu", torch.float32, seed=3, tp=tp,
                                          max_positions=64)
        assert m.hq == CFG.num_attention_heads // world and m.hkv == CFG.num_key_value_heads // world
        out = _run(m, ids)
        if rank == 0:
            q.put(out)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tp_decode_matches_tp1_on_gloo(world):
    torch.manual_seed(0)
    ids = torch.randint(0, CFG.vocab_size, (3, 6))
    ref = _run(Llama3DecodeModel.random_init(CFG, "cpu", torch.float32, seed=3, max_positions=64),
               ids)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, ids, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-5)


def test_shard_layout_matches_reference():
    """Column shard i = rows [i*o/N, (i+1)*o/N); row shard i = columns (reference
    tests/test_tensor_parallel.py:14-15,31-32); partial products sum to the dense one."""
    torch.manual_seed(31)
    x = torch.randn(2, 3, 8)
    w = torch.randn(6, 8)
    cols = torch.cat([x @ shard_rows(w, r, 2).T for r in range(2)], -1)
    torch.testing.assert_close(cols, x @ w.T, rtol=1e-6, atol=1e-6)
    w2 = torch.randn(5, 8)
    parts = sum(x[..., r * 4:(r + 1) * 4] @ shard_cols(w2, r, 2).T for r in range(2))
    torch.testing.assert_close(parts, x @ w2.T, rtol=1e-6, atol=1e-6)


def _dying_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        os._exit(3)          # a rank that leaves between steps, no collective in flight
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        q.put("completed")
    except Exception as e:   # the survivor learns through a timed-out collective
        q.put("error:" + type(e).__name__)


def test_dead_rank_is_detected_by_timeout():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    msg = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert msg.startswith("error:"), msg
    assert procs[1].exitcode == 3
