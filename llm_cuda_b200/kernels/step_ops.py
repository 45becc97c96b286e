"""Decode-step kernels around the attention path (CUDA): tcgen05 decode GEMM,
fused residual-add + RMSNorm, SwiGLU.

``add_rmsnorm`` replaces the residual add (``src/llm_cuda/models/llama3/model.py:37,42``
of llm-cuda) plus ``RMSNorm.forward`` (``norm.py:31-33``); ``swiglu`` replaces
``triton_swiglu`` (``kernels/triton/swiglu.py:103-107``).  Both run in the C-ABI
library; there is no fallback.
"""

from __future__ import annotations

import torch

from .. import _native as N


def add_rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float,
                delta: torch.Tensor | None = None, out: torch.Tensor | None = None):
    """In place ``x += delta`` (if given); returns ``rmsnorm(x) * weight``.
    ``x`` must be contiguous ``[..., hidden]`` (it is updated in place)."""
    if not x.is_contiguous():
        raise ValueError("x must be contiguous (updated in place)")
    hidden = x.shape[-1]
    rows = x.numel() // hidden
    if delta is not None:
        delta = delta.contiguous()
        if delta.shape != x.shape or delta.dtype != x.dtype:
            raise ValueError("delta must match x")
    w = weight if weight.dtype == x.dtype else weight.to(x.dtype)
    out = torch.empty_like(x) if out is None else out
    rc = N.load().llmc_add_rmsnorm(x.data_ptr(), N.ptr(delta), w.contiguous().data_ptr(),
                                   out.data_ptr(), rows, hidden, float(eps),
                                   N.dtype_code(x.dtype), N.stream_handle(x.device))
    N.check(rc, "llmc_add_rmsnorm")
    return out


def swiglu(gate_up: torch.Tensor) -> torch.Tensor:
    """``silu(g) * u`` for ``gate_up [..., 2*inter] = [g | u]`` -> ``[..., inter]``."""
    gate_up = gate_up.contiguous()
    inter = gate_up.shape[-1] // 2
    rows = gate_up.numel() // (2 * inter)
    out = gate_up.new_empty(*gate_up.shape[:-1], inter)
    rc = N.load().llmc_swiglu(gate_up.data_ptr(), out.data_ptr(), rows, inter,
                              N.dtype_code(gate_up.dtype), N.stream_handle(gate_up.device))
    N.check(rc, "llmc_swiglu")
    return out


_gemm_ws: dict = {}


def _gemm_workspace(device: torch.device, Mb: int, n_out: int, k: int):
    """fp32 partial slots + int32 counters (kept zero by the kernel) for one shape."""
    key = (device.index, Mb, n_out, k)
    ws = _gemm_ws.get(key)
    if ws is None:
        nbytes = N.load().llmc_decode_gemm_workspace_bytes(Mb, n_out, k)
        ws = (torch.empty(max(nbytes // 4, 1), dtype=torch.float32, device=device),
              torch.zeros(n_out // 128, dtype=torch.int32, device=device))
        _gemm_ws[key] = ws
    return ws


def decode_gemm(x: torch.Tensor, w: torch.Tensor, status: torch.Tensor | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """``y = x @ w.T`` on the tcgen05 tensor cores for decode batches (bf16, rows of
    ``x`` <= 256, ``w`` [N, K] with N % 128 == 0 and K % 64 == 0)."""
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        raise ValueError("decode_gemm takes bf16 x and W")
    K = x.shape[-1]
    x2 = x.reshape(-1, K).contiguous()
    Mb, n_out = x2.shape[0], w.shape[0]
    y = torch.empty(Mb, n_out, dtype=torch.bfloat16, device=x.device) if out is None else out
    ws, cnt = _gemm_workspace(x.device, Mb, n_out, K)
    if status is None:
        from .decode_attention import default_status

        status = default_status(x.device)
    rc = N.load().llmc_decode_gemm(x2.data_ptr(), w.data_ptr(), y.data_ptr(), ws.data_ptr(),
                                   ws.numel() * 4, cnt.data_ptr(), Mb, n_out, K, status.data_ptr(),
                                   N.stream_handle(x.device))
    N.check(rc, "llmc_decode_gemm")
    return y.view(*x.shape[:-1], n_out)


_argmax_ws: dict = {}


def argmax_rows(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """``torch.argmax(x, dim=-1)`` of a 2-D CUDA tensor in one launch (the greedy pick
    of the decode loop, ``model.py:214``): first index of the maximum, int64."""
    if x.dim() != 2:
        raise ValueError("argmax_rows takes a 2-D tensor")
    x = x.contiguous()
    rows, n = x.shape
    out = torch.empty(rows, dtype=torch.int64, device=x.device) if out is None else out
    key = (x.device.index, rows)
    ws = _argmax_ws.get(key)
    if ws is None:   # zero once; the kernel leaves it at zero
        nbytes = N.load().llmc_argmax_workspace_bytes(rows)
        ws = torch.zeros(max((nbytes + 7) // 8, 1), dtype=torch.int64, device=x.device)
        _argmax_ws[key] = ws
    rc = N.load().llmc_argmax(x.data_ptr(), out.data_ptr(), rows, n, N.dtype_code(x.dtype),
                              ws.data_ptr(), N.stream_handle(x.device))
    N.check(rc, "llmc_argmax")
    return out
