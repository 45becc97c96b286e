"""tcgen05 decode GEMM against a plain PyTorch fp32 matmul."""

import pytest
import torch

from llm_cuda_b200 import _native as N
from llm_cuda_b200.kernels.step_ops import decode_gemm

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("Mb,n_out,k", [
    (64, 128, 64),            # one tile, one k-chunk
    (64, 256, 4096),          # two tiles split over many CTAs (stream-K reduction)
    (64, 6144, 4096),         # q/k/v projection of Llama-3-8B
    (64, 4096, 14336),        # down_proj
    (64, 28672, 4096),        # gate/up: more tiles than SMs, tiles shared at range edges
    (64, 1536, 4096),         # q/k/v of one rank at TP4
    (64, 768, 4096),          # q/k/v of one rank at TP8 (clusters of 8)
    (64, 4096, 512),          # o_proj of one rank at TP8
    (64, 3584, 4096),         # gate/up of one rank at TP8
    (128, 512, 1024),         # 128-row batch tile
    (256, 256, 512),          # 256-row batch tile
])
def test_decode_gemm_matches_fp32(Mb, n_out, k):
    g = torch.Generator(device=DEV).manual_seed(Mb + n_out + k)
    x = torch.randn(Mb, k, device=DEV, generator=g).bfloat16()
    w = (0.02 * torch.randn(n_out, k, device=DEV, generator=g)).bfloat16()
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    ref = x.float() @ w.float().T
    for _ in range(2):   # the tile counters must come back to zero after every call
        y = decode_gemm(x, w, status=status)
        torch.cuda.synchronize()
        N.raise_on_status(status)
        assert torch.isfinite(y.float()).all()
        torch.testing.assert_close(y.float(), ref, rtol=1e-2, atol=2e-2)
    from llm_cuda_b200.kernels.step_ops import _gemm_workspace
    _, cnt = _gemm_workspace(DEV, Mb, n_out, k)
    assert torch.count_nonzero(cnt) == 0
