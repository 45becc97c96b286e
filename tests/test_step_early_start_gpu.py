"""Early start of the attention launch (LLMC_DECODE_EARLY_TABLES) in the decode step.

With the flag, each layer's attention launch scans the lengths and starts streaming K/V
before the QKV projection that precedes it has finished (programmatic dependent launch;
the projection runs on the tcgen05 GEMM, which lets dependents start early).  The steps
must be bit-identical to the steps without it, eager and graphed.
"""

import pytest
import torch

from llm_cuda_b200.models.llama3.decode_model import DecodeConfig, DecodeGraph, Llama3DecodeModel

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def test_early_tables_step_equals_ordered_step():
    """Attention launches that start their K/V stream before the QKV projection ends
    (LLMC_DECODE_EARLY_TABLES) give bit-identical steps, eager and graphed."""
    cfg = DecodeConfig(vocab_size=1000, hidden_size=512, intermediate_size=1024,
                       num_hidden_layers=3, num_attention_heads=8, num_key_value_heads=2)
    m = Llama3DecodeModel.random_init(cfg, DEV, torch.bfloat16, seed=11, max_positions=512)
    m.tc_projections = {"qkv", "o", "gate_up", "down"}     # PDL-aware GEMMs before attention
    B, S, steps = 64, 300, 4
    ids = torch.randint(0, cfg.vocab_size, (B, S), generator=torch.Generator().manual_seed(3)).to(DEV)

    def run(early: bool, graph: bool):
        m.early_tables = early
        cache = m.make_cache(B, 512, page_size=16, shuffle_seed=5)
        nxt = m.prefill(ids, cache).argmax(-1)
        out = []
        if graph:
            gr = DecodeGraph(m, cache, nxt, partition_tokens=0)
            for _ in range(steps):
                gr.replay()
                out.append(gr.logits.clone())
        else:
            for _ in range(steps):
                lg = m.decode_step(nxt, cache, partition_tokens=0)
                out.append(lg.clone())
                nxt = lg.argmax(-1)
        torch.cuda.synchronize()
        m.check_status(cache)
        return torch.stack(out)

    ref = run(False, False)
    assert torch.equal(run(True, False), ref)
    assert torch.equal(run(True, True), ref)
    m.early_tables = True
