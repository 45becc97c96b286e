"""Fused residual-add + RMSNorm and SwiGLU kernels for the decode step (CUDA).

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
