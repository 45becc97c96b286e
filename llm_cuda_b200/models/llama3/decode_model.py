"""Llama 3 decode step with KV-head-sharded tensor parallelism (config 5 harness).

The caller of the decode-attention path: one decode step of a Llama-3 model
(``src/llm_cuda/models/llama3/model.py:14-107,178-218`` of llm-cuda) with

* the attention hot path as ONE launch per layer: the fused decode kernel
  (``llmc_rope_append_decode_strided``) rotates the new token's q/k, appends k/v to
  the pages and attends over the whole context with the balanced split and its
  in-kernel merge, reading q/k/v in place from the QKV projection output — instead
  of ``build_rope_cache`` / ``apply_rotary`` / ``append`` / ``get_kv`` /
  ``triton_decode_attention`` (``attention.py:100-150``);
* tensor parallelism over ranks, one process per GPU.  Shards follow the
  reference's layout (``parallel/tensor_parallel.py:8-90``): q/k/v/gate/up are
  column-split (rank i owns output rows ``[i*o/N, (i+1)*o/N)``, i.e. whole query
  and KV heads), o_proj/down_proj are row-split (input columns), and the
  reference's in-process sum of row-parallel partials (:83-90) is an all-reduce
  over NVLink: this package's fused kernel (``enable_fused_allreduce``: one launch
  that also does the residual add + RMSNorm, one- or two-shot over peer memory) or
  NCCL.  Embedding and lm_head are replicated (the reference does not shard them,
  model.py:50,115);
* residual add + RMSNorm (``norm.py:31-33``), SwiGLU (``kernels/triton/swiglu.py:103-107``)
  and the greedy argmax as CUDA kernels of this package; dense projections on cuBLAS
  or the tcgen05 decode GEMM (``tc_projections``).

``decode_step`` allocates nothing and reads lengths on the device, so the whole
step (all layers, all-reduces, lm_head, greedy argmax) is captured once in a
CUDA graph and replayed per token (``DecodeGraph``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from ...kernels.step_ops import add_rmsnorm, argmax_rows, decode_gemm, swiglu
from .kv_cache import PagedKVCache, make_block_table
from .rotary import RopeTable


# Layer projections of the decode step served by the tcgen05 decode GEMM by default.
# Measured at B=64 in CUDA graphs of back-to-back calls with weights larger than L2,
# cuBLAS is ahead on the full-size layer shapes (qkv 11.9 vs 14.9 us, gate_up 42.5 vs
# 50.8 us), so none are by default at TP1-2; the vocabulary projection (lm_head) always
# uses the tcgen05 GEMM (176 vs 184 us).  On one rank's q/k/v at TP >= 4 the tcgen05
# GEMM is ahead (1536 x 4096: 6.8 vs 8.2 us; 768 x 4096: 5.4 vs 7.8 us), and it lets
# the attention launch after it start early (programmatic dependent launch).
DEFAULT_TC_PROJECTIONS = ()
TC_PROJECTIONS_TP4_UP = ("qkv",)


@dataclass
class DecodeConfig:
    vocab_size: int = 128256
    hidden_size: int = 4096
    intermediate_size: int = 14336
    num_hidden_layers: int = 32
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    rope_theta: float = 500000.0
    rms_norm_eps: float = 1e-5
    initializer_range: float = 0.02

    @property
    def head_dim(self) -> int:  # config.py:40-42 of the reference
        return self.hidden_size // self.num_attention_heads


class TensorParallel:
    """Rank/size of the TP group and its all-reduce (identity when size == 1).

    ``fused`` (an ``NvlinkAllReduce``, set by ``Llama3DecodeModel.enable_fused_allreduce``)
    takes the decode rows' all-reduce + residual add + RMSNorm in one kernel; rows it
    does not take (prefill) use ``all_reduce_`` (NCCL).
    """

    def __init__(self, rank: int = 0, size: int = 1, group=None):
        self.rank, self.size, self.group = rank, size, group
        self.fused = None

    def all_reduce_(self, x: torch.Tensor) -> torch.Tensor:
        if self.size > 1:
            import torch.distributed as dist

            dist.all_reduce(x, group=self.group)
        return x


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """``x * rsqrt(mean(x^2) + eps) * w`` in the tensor dtype (norm.py:31-33)."""
    var = x.pow(2).mean(dim=-1, keepdim=True)
    return x * torch.rsqrt(var + eps) * w


def shard_rows(w: torch.Tensor, rank: int, size: int) -> torch.Tensor:
    """Column-parallel shard: output rows of rank ``rank`` (tensor_parallel.py:44-49)."""
    n = w.shape[0] // size
    return w[rank * n:(rank + 1) * n]


def shard_cols(w: torch.Tensor, rank: int, size: int) -> torch.Tensor:
    """Row-parallel shard: input columns of rank ``rank`` (tensor_parallel.py:83-88)."""
    n = w.shape[1] // size
    return w[:, rank * n:(rank + 1) * n]


class Llama3DecodeModel:
    def __init__(self, cfg: DecodeConfig, device, dtype=torch.bfloat16,
                 tp: TensorParallel | None = None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype
        self.tp = tp or TensorParallel()
        N = self.tp.size
        if cfg.num_key_value_heads % N or cfg.num_attention_heads % N or cfg.intermediate_size % N:
            raise ValueError("heads and intermediate size must divide by the TP size")
        self.hq = cfg.num_attention_heads // N
        self.hkv = cfg.num_key_value_heads // N
        self.inter = cfg.intermediate_size // N
        self.layers: list[dict] = []
        self.embed = None
        self.final_norm = None
        self.lm_head = None
        self.rope: RopeTable | None = None
        # Optional replacement of the attention core ``(layer, q, k, v, layer_cache) -> out``
        # taking the raw (un-rotated) q/k/v; tests of the TP plumbing on CPU ranks use it.
        self.attn_core = None
        # Decode projections that run on the tcgen05 decode GEMM (the rest: F.linear).
        self.tc_projections = set(DEFAULT_TC_PROJECTIONS if N < 4 else TC_PROJECTIONS_TP4_UP)
        # Optional ``mark(phase)`` called after each phase of ``decode_step`` (profiling:
        # e.g. records a timing event; phases are named in ``decode_step``).
        self.mark = None
        # Attention launches may start their K/V stream before the previous kernel ends
        # (LLMC_DECODE_EARLY_TABLES): nothing else in the step writes a layer's tables.
        self.early_tables = True

    def _mark(self, phase: str) -> None:
        if self.mark is not None:
            self.mark(phase)

    def check_status(self, cache: PagedKVCache) -> None:
        """Synchronise and raise if a kernel of the step (attention, or the fused
        all-reduce at TP > 1) reported an error through its status word."""
        cache.check_status()
        if self.tp.fused is not None:
            self.tp.fused.check_status()

    # -- weights ---------------------------------------------------------------
    def _add_layer(self, full: dict) -> None:
        """Shard one layer given its FULL (unsharded) reference-named weights."""
        r, N = self.tp.rank, self.tp.size
        wq = shard_rows(full["q_proj"], r, N)
        wk = shard_rows(full["k_proj"], r, N)
        wv = shard_rows(full["v_proj"], r, N)
        wg = shard_rows(full["gate_proj"], r, N)
        wu = shard_rows(full["up_proj"], r, N)
        to = dict(device=self.device, dtype=self.dtype)
        self.layers.append({
            "in_norm": full["input_layernorm"].to(**to),
            "wqkv": torch.cat([wq, wk, wv], 0).to(**to).contiguous(),
            "wo": shard_cols(full["o_proj"], r, N).to(**to).contiguous(),
            "post_norm": full["post_attention_layernorm"].to(**to),
            "wgu": torch.cat([wg, wu], 0).to(**to).contiguous(),
            "wdown": shard_cols(full["down_proj"], r, N).to(**to).contiguous(),
        })

    def _finish(self, embed, final_norm, lm_head, max_positions: int) -> None:
        to = dict(device=self.device, dtype=self.dtype)
        self.embed = embed.to(**to).contiguous()
        self.final_norm = final_norm.to(**to)
        self.lm_head = lm_head.to(**to).contiguous()
        self.rope = RopeTable(max_positions, self.cfg.head_dim, self.cfg.rope_theta, self.device,
                              self.dtype)

    @classmethod
    def random_init(cls, cfg: DecodeConfig, device, dtype=torch.bfloat16, seed: int = 0,
                    tp: TensorParallel | None = None, max_positions: int = 8192):
        """Seeded N(0, initializer_range) weights (model.py:122-139); norm weights are ones.
        Every rank draws the same full layer on its own GPU and keeps its shard."""
        m = cls(cfg, device, dtype, tp)
        H, I, d = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
        shapes = {"q_proj": (cfg.num_attention_heads * d, H), "k_proj": (cfg.num_key_value_heads * d, H),
                  "v_proj": (cfg.num_key_value_heads * d, H), "o_proj": (H, cfg.num_attention_heads * d),
                  "gate_proj": (I, H), "up_proj": (I, H), "down_proj": (H, I)}
        std = cfg.initializer_range
        for li in range(cfg.num_hidden_layers):
            g = torch.Generator(device=m.device).manual_seed(seed * 1000003 + li)
            full = {k: torch.empty(s, device=m.device, dtype=dtype).normal_(0.0, std, generator=g)
                    for k, s in shapes.items()}
            full["input_layernorm"] = torch.ones(H)
            full["post_attention_layernorm"] = torch.ones(H)
            m._add_layer(full)
            del full
        g = torch.Generator(device=m.device).manual_seed(seed * 1000003 + 999983)
        embed = torch.empty(cfg.vocab_size, H, device=m.device, dtype=dtype).normal_(0.0, std, generator=g)
        head = torch.empty(cfg.vocab_size, H, device=m.device, dtype=dtype).normal_(0.0, std, generator=g)
        m._finish(embed, torch.ones(H), head, max_positions)
        return m

    @classmethod
    def from_reference_state_dict(cls, cfg: DecodeConfig, sd: dict, device, dtype,
                                  tp: TensorParallel | None = None, max_positions: int = 8192):
        """Load a full (tp_size = 1) reference ``Llama3ForCausalLM.state_dict()``."""
        m = cls(cfg, device, dtype, tp)
        for li in range(cfg.num_hidden_layers):
            p = f"model.layers.{li}."
            m._add_layer({
                "q_proj": sd[p + "self_attn.q_proj.weight"], "k_proj": sd[p + "self_attn.k_proj.weight"],
                "v_proj": sd[p + "self_attn.v_proj.weight"], "o_proj": sd[p + "self_attn.o_proj.weight"],
                "gate_proj": sd[p + "mlp.gate_proj.weight"], "up_proj": sd[p + "mlp.up_proj.weight"],
                "down_proj": sd[p + "mlp.down_proj.weight"],
                "input_layernorm": sd[p + "input_layernorm.weight"],
                "post_attention_layernorm": sd[p + "post_attention_layernorm.weight"],
            })
        m._finish(sd["model.embed_tokens.weight"], sd["model.norm.weight"], sd["lm_head.weight"],
                  max_positions)
        return m

    # -- cache -----------------------------------------------------------------
    def make_cache(self, batch: int, max_seq_len: int, page_size: int = 16,
                   shuffle_seed: int | None = None) -> PagedKVCache:
        """Paged cache for this rank's KV heads; pages drawn from the pool in random
        order when ``shuffle_seed`` is given."""
        max_pages = math.ceil(max_seq_len / page_size)
        bt = None
        num_pages = None
        if shuffle_seed is not None:
            num_pages = batch * max_pages
            bt = make_block_table(batch, max_pages, num_pages, max_pages,
                                  generator=torch.Generator().manual_seed(shuffle_seed))
        return PagedKVCache.create(self.cfg.num_hidden_layers, self.hkv, self.cfg.head_dim,
                                   max_seq_len, page_size, self.device, self.dtype,
                                   batch_size=batch, num_pages=num_pages, block_table=bt)

    # -- forward pieces --------------------------------------------------------
    def _split_qkv(self, qkv: torch.Tensor, B: int, S: int):
        d = self.cfg.head_dim
        q, k, v = qkv.split([self.hq * d, self.hkv * d, self.hkv * d], dim=-1)
        # [B, S, H*d] -> [B, H, S, d] (attention.py:52-54)
        q = q.view(B, S, self.hq, d).transpose(1, 2)
        k = k.view(B, S, self.hkv, d).transpose(1, 2)
        v = v.view(B, S, self.hkv, d).transpose(1, 2)
        return q, k, v

    def _mlp(self, L: dict, x: torch.Tensor, mark=None) -> torch.Tensor:
        mark = mark or (lambda _: None)
        gu = self._linear(x, L["wgu"], "gate_up")
        mark("gemm_gate_up")
        if gu.is_cuda:
            h = swiglu(gu)                                 # fused CUDA kernel
        else:
            gate, up = gu.split(self.inter, dim=-1)
            h = (gate * torch.sigmoid(gate)) * up         # swiglu.py:103-107
        mark("swiglu")
        out = self._linear(h, L["wdown"], "down")    # row-parallel partial
        mark("gemm_down")
        return out

    def _linear(self, x: torch.Tensor, w: torch.Tensor, name: str) -> torch.Tensor:
        """``x @ w.T`` for the projection ``name``: the tcgen05 decode GEMM when ``name``
        is in ``self.tc_projections`` and the shape qualifies, else ``F.linear``."""
        K = x.shape[-1]
        rows = x.numel() // K
        if (name in self.tc_projections and x.is_cuda and x.dtype == torch.bfloat16
                and rows <= 256 and w.shape[0] % 128 == 0 and K % 64 == 0):
            return decode_gemm(x.reshape(rows, K), w).view(*x.shape[:-1], w.shape[0])
        return F.linear(x, w)

    def _lm_head(self, h: torch.Tensor) -> torch.Tensor:
        """Vocabulary projection.  At decode batch sizes the 1 GB bf16 weight streams
        through the tcgen05 decode GEMM (persistent stream-K, TMEM accumulators), which
        is faster than cuBLAS on this shape; other dtypes/shapes use F.linear."""
        if (h.is_cuda and h.dtype == torch.bfloat16 and h.shape[0] <= 256
                and self.lm_head.shape[0] % 128 == 0 and h.shape[-1] % 64 == 0):
            return decode_gemm(h, self.lm_head)
        return F.linear(h, self.lm_head)

    def enable_fused_allreduce(self, rows_cap: int) -> None:
        """Serve the all-reduce + residual add + RMSNorm of up to ``rows_cap`` decode
        rows with the one-shot NVLink kernel (every rank of the group must call it)."""
        from ...kernels.allreduce import NvlinkAllReduce

        if self.tp.size > 1 and self.tp.fused is None:
            self.tp.fused = NvlinkAllReduce(self.tp.group, self.tp.rank, self.tp.size, rows_cap,
                                            self.cfg.hidden_size, self.dtype, self.device)

    def _reduce_add_norm(self, x: torch.Tensor, w: torch.Tensor, partial: torch.Tensor | None):
        """All-reduce of a row-parallel ``partial`` (tensor_parallel.py:83-90), residual
        add and RMSNorm: returns ``(x, h)``.  The fused NVLink kernel takes it when
        enabled and the rows fit; otherwise NCCL + the add/norm kernel."""
        if partial is None:
            return self._add_norm(x, w, None)
        f = self.tp.fused
        if f is not None and f.supports(x) and x.is_contiguous():
            return x, f.add_rmsnorm(partial.contiguous(), x, w, self.cfg.rms_norm_eps)
        return self._add_norm(x, w, self.tp.all_reduce_(partial))

    def _add_norm(self, x: torch.Tensor, w: torch.Tensor, delta: torch.Tensor | None):
        """Residual add (model.py:37,42) + RMSNorm (norm.py:31-33): returns ``(x, h)``.
        On CUDA one fused kernel updates ``x`` in place; the CPU branch serves only the
        CPU-rank tests of the TP plumbing."""
        if x.is_cuda:
            return x, add_rmsnorm(x, w, self.cfg.rms_norm_eps, delta=delta)
        if delta is not None:
            x = x + delta
        return x, rms_norm(x, w, self.cfg.rms_norm_eps)

    def prefill(self, ids: torch.Tensor, cache: PagedKVCache) -> torch.Tensor:
        """Process prompts ``ids [B, S]`` into an EMPTY cache; returns last-token logits.

        Prompt attention (off the decode path) is causal SDPA over the rotated q/k;
        the S tokens' k/v go into the pages with the fused RoPE + append kernel.
        """
        cfg = self.cfg
        B, S = ids.shape
        x = F.embedding(ids, self.embed).contiguous()
        delta = None
        for li, L in enumerate(self.layers):
            lc = cache.get_layer(li)
            x, h = self._reduce_add_norm(x, L["in_norm"], delta)
            q, k, v = self._split_qkv(F.linear(h, L["wqkv"]), B, S)
            q_rot = lc.append_rotary(q, k, v, self.rope)
            kc, vc = lc.get_kv()                             # rotated k as stored
            rep = self.hq // self.hkv
            attn = F.scaled_dot_product_attention(
                q_rot, kc.repeat_interleave(rep, dim=1), vc.repeat_interleave(rep, dim=1),
                is_causal=True)
            attn = attn.transpose(1, 2).reshape(B, S, self.hq * cfg.head_dim)
            x, h = self._reduce_add_norm(x, L["post_norm"], F.linear(attn, L["wo"]))
            delta = self._mlp(L, h)
        x, h = self._reduce_add_norm(x, self.final_norm, delta)
        return F.linear(h[:, -1], self.lm_head)

    def decode_step(self, ids: torch.Tensor, cache: PagedKVCache,
                    partition_tokens: int | None = None) -> torch.Tensor:
        """One token per sequence: ``ids [B]`` -> logits ``[B, vocab]``."""
        cfg = self.cfg
        B = ids.shape[0]
        mark = self._mark
        x = F.embedding(ids.view(B, 1), self.embed)          # [B, 1, H]
        mark("embed")
        delta = None
        for li, L in enumerate(self.layers):
            lc = cache.get_layer(li)
            x, h = self._reduce_add_norm(x, L["in_norm"], delta)
            mark("allreduce_add_norm" if delta is not None else "add_norm")
            q, k, v = self._split_qkv(self._linear(h, L["wqkv"], "qkv"), B, 1)
            mark("gemm_qkv")
            if self.attn_core is not None:
                attn = self.attn_core(li, q, k, v, lc)
            else:
                # RoPE + page append + paged attention in one fused decode launch.  A
                # layer's lengths, block table and pages are written only by its own
                # attention launch (and the host between steps), so the K/V stream may
                # start before the QKV projection has finished.
                attn = lc.rope_append_decode(q, k, v, self.rope,
                                             partition_tokens=partition_tokens,
                                             early_tables=self.early_tables)
            mark("attention")
            attn = attn.reshape(B, 1, self.hq * cfg.head_dim)
            partial = self._linear(attn, L["wo"], "o")
            mark("gemm_o")
            x, h = self._reduce_add_norm(x, L["post_norm"], partial)
            mark("allreduce_add_norm")
            delta = self._mlp(L, h, mark)
        x, h = self._reduce_add_norm(x, self.final_norm, delta)
        mark("allreduce_add_norm")
        logits = self._lm_head(h[:, 0])
        mark("lm_head")
        return logits

    def bytes_per_step(self, cache: PagedKVCache) -> tuple[int, int]:
        """(weight bytes, KV bytes) this rank reads in one decode step at the current
        lengths (KV after the step's append)."""
        esz = torch.finfo(self.dtype).bits // 8
        w = sum(t.numel() for L in self.layers for t in (L["wqkv"], L["wo"], L["wgu"], L["wdown"]))
        w = (w + self.lm_head.numel()) * esz
        lens = cache.get_layer(0).host_lengths
        kv = sum(x + 1 for x in lens) * self.hkv * self.cfg.head_dim * 2 * esz * len(self.layers)
        return w, kv


class DecodeGraph:
    """The whole greedy decode step captured once: ``ids -> logits -> argmax -> ids``.

    ``replay()`` advances every sequence by one token with no host work besides the
    launch; the cache's host length mirrors are advanced to match.
    """

    def __init__(self, model: Llama3DecodeModel, cache: PagedKVCache, ids: torch.Tensor,
                 partition_tokens: int):
        self.model, self.cache = model, cache
        self.ids = ids.clone()
        self.next_ids = torch.empty_like(self.ids)
        self.logits = None
        # warm-up (allocates workspaces outside the capture), then undo its append
        lens0 = cache.get_layer(0).seq_lens.clone()
        host0 = list(cache.get_layer(0).host_lengths)
        warm = model.decode_step(self.ids, cache, partition_tokens)
        argmax_rows(warm)                       # its workspace exists before the capture
        torch.cuda.synchronize()
        self._reset(lens0, host0)
        s = torch.cuda.Stream(device=model.device)
        s.wait_stream(torch.cuda.current_stream(model.device))
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(self.graph, stream=s):
                model._mark("start")
                self.logits = model.decode_step(self.ids, cache, partition_tokens)
                argmax_rows(self.logits, out=self.next_ids)
                self.ids.copy_(self.next_ids)
                model._mark("argmax")
        torch.cuda.current_stream(model.device).wait_stream(s)
        torch.cuda.synchronize()
        self._reset(lens0, host0)

    def _reset(self, lens0, host0):
        for lc in self.cache.layer_caches:
            lc.seq_lens.copy_(lens0)
            lc.host_lengths = list(host0)

    def replay(self) -> None:
        self.graph.replay()
        for lc in self.cache.layer_caches:
            lc.advance_host_lengths(1)
