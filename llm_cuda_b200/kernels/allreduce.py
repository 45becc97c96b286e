"""One-shot NVLink all-reduce fused with the residual add and RMSNorm (TP decode).

Replaces, for the decode rows of a tensor-parallel step, the NCCL all-reduce of the
row-parallel o_proj / down_proj partials (the in-process sum of
``src/llm_cuda/parallel/tensor_parallel.py:83-90`` of llm-cuda) and the residual add +
RMSNorm that follows it (``models/llama3/model.py:37-42``, ``norm.py:31-33``) with one
kernel per call (``llmc_allreduce_add_rmsnorm``).  Each rank's receive
region is a plain device allocation shared through a CUDA IPC handle, exchanged once
over the process group; the kernel pushes each row to the peers as 8-byte words that
carry their own epoch, so a receiver knows a word has arrived without any fence or
separate flag (bounded waits, no multicast).
"""

from __future__ import annotations

import ctypes

import torch

from .. import _native as N


class NvlinkAllReduce:
    """Shared regions of one rank and the fused all-reduce + add + RMSNorm over them.

    Build it on every rank of ``group`` with the same ``rows_cap``/``hidden``/``dtype``;
    calls must then be issued in the same order on all ranks.  ``close()`` (after a
    barrier) releases the mappings.
    """

    def __init__(self, group, rank: int, world: int, rows_cap: int, hidden: int,
                 dtype: torch.dtype, device: torch.device):
        import torch.distributed as dist

        if not 1 <= world <= 8:
            raise ValueError("the fused all-reduce supports 1 to 8 ranks")
        self.lib = N.load()
        self.rank, self.world, self.rows_cap, self.hidden = rank, world, rows_cap, hidden
        self.dtype, self.device = dtype, torch.device(device)
        dt = N.dtype_code(dtype)
        fb = ctypes.c_size_t(0)
        with torch.cuda.device(self.device):
            rb = self.lib.llmc_ar_region_bytes(world, rows_cap, hidden, dt, ctypes.byref(fb))
            if fb.value:
                raise RuntimeError("llmc_ar_region_bytes asks for a flag region this binding "
                                   "does not allocate")
            hsz = self.lib.llmc_ipc_handle_bytes()
            ptr = ctypes.c_void_p()
            h = ctypes.create_string_buffer(hsz)
            N.check(self.lib.llmc_ipc_alloc(rb, ctypes.byref(ptr), h), "llmc_ipc_alloc")
            self._own = [ptr.value]
            gathered = [None] * world
            dist.all_gather_object(gathered, h.raw, group=group)
            self._opened = []
            recv = []
            for q in range(world):
                if q == rank:
                    recv.append(self._own[0])
                    continue
                hq = gathered[q]
                ptr = ctypes.c_void_p()
                N.check(self.lib.llmc_ipc_open(ctypes.create_string_buffer(hq, len(hq)),
                                               ctypes.byref(ptr)), "llmc_ipc_open")
                self._opened.append(ptr.value)
                recv.append(ptr.value)
        self.recv_ptrs = torch.tensor(recv, dtype=torch.int64, device=self.device)
        self.epoch = torch.zeros(rows_cap, dtype=torch.int32, device=self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.failed = False     # set once a wait timeout has been reported
        dist.barrier(group=group)   # every rank has mapped every region before first use

    def supports(self, x: torch.Tensor) -> bool:
        rows = x.numel() // x.shape[-1]
        return (x.is_cuda and x.dtype == self.dtype and x.shape[-1] == self.hidden
                and rows <= self.rows_cap)

    def add_rmsnorm(self, partial: torch.Tensor, x: torch.Tensor, weight: torch.Tensor,
                    eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
        """``x += all_reduce(partial)`` in place; returns ``rmsnorm(x) * weight``."""
        if self.failed:
            raise N.DeviceStatusError(
                "NvlinkAllReduce: a previous call timed out waiting for a peer; the ranks' "
                "epochs are out of step, so this instance refuses further calls (rebuild it)")
        if not (x.is_contiguous() and partial.is_contiguous()):
            raise ValueError("x and partial must be contiguous")
        rows = x.numel() // self.hidden
        w = weight if weight.dtype == x.dtype else weight.to(x.dtype)
        out = torch.empty_like(x) if out is None else out
        rc = self.lib.llmc_allreduce_add_rmsnorm(
            partial.data_ptr(), self.recv_ptrs.data_ptr(), None,
            self.epoch.data_ptr(), x.data_ptr(), w.contiguous().data_ptr(), out.data_ptr(),
            self.status.data_ptr(), self.rank, self.world, rows, self.rows_cap, self.hidden,
            float(eps), N.dtype_code(x.dtype), N.stream_handle(x.device))
        N.check(rc, "llmc_allreduce_add_rmsnorm")
        return out

    def check_status(self) -> None:
        """Synchronise and raise ``DeviceStatusError`` if a call timed out; after that the
        instance refuses further calls."""
        try:
            N.raise_on_status(self.status)
        except N.DeviceStatusError:
            self.failed = True
            # Keep the timeout bit set: kernels already captured in a graph then return
            # at once on replay instead of each waiting out the deadline.
            self.status.fill_(N.LLMC_STATUS_WAIT_TIMEOUT)
            raise

    def close(self) -> None:
        """Unmap the peers' regions and free this rank's (call after a barrier)."""
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            for ptr in self._opened:
                self.lib.llmc_ipc_close(ctypes.c_void_p(ptr))
            for ptr in self._own:
                self.lib.llmc_ipc_free(ctypes.c_void_p(ptr))
        self._opened, self._own = [], []
