"""ctypes binding of the C ABI in ``include/llm_cuda_b200.h``.

The shared library is built in-tree by ``llm_cuda_b200.build`` into
``llm_cuda_b200/_lib/libllmcuda_b200.so``.  There is no fallback: if the library
is missing, every kernel entry point raises ``NativeLibraryError``.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libllmcuda_b200.so")

LLMC_F32, LLMC_F16, LLMC_BF16 = 0, 1, 2
LLMC_DECODE_FORCE_GENERIC = 1
LLMC_DECODE_EARLY_TABLES = 2
LLMC_STATUS_WAIT_TIMEOUT = 1

STATUS_BITS = {
    1: "pipeline wait timeout",
    2: "block-table page id out of range",
    4: "append past the cache capacity",
    8: "RoPE position outside the cos/sin table",
    16: "sequence length larger than the block table can address",
}

_DTYPE_CODE = {torch.float32: LLMC_F32, torch.float16: LLMC_F16, torch.bfloat16: LLMC_BF16}

# (name, restype, argtypes) of every exported symbol.
_P, _I, _F, _SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
SIGNATURES = {
    "llmc_rope_append": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P] + [_I] * 10 + [_P, _P]),
    "llmc_decode_partials_bytes": (_SZ, [_I, _I, _I, _I, ctypes.POINTER(_SZ)]),
    "llmc_num_partitions": (_I, [_I, _I]),
    "llmc_balanced_partials_bytes": (_SZ, [_I, _I, _I, _I, ctypes.POINTER(_SZ)]),
    "llmc_decode_balanced_supported": (_I, [_P, _P, _P] + [_I] * 5),
    "llmc_paged_decode": (_I, [_P] * 9 + [_I] * 8 + [_F, _I, _I, _P]),
    "llmc_lse_merge": (_I, [_P, _P, _P, _P] + [_I] * 6 + [_P]),
    "llmc_paged_decode_noalloc": (_I, [_P] * 7 + [_I] * 8 + [_F, _I, _P]),
    "llmc_paged_decode_noalloc_capacity_bytes": (_SZ, []),
    "llmc_rope_append_decode": (_I, [_P] * 10 + [_I] + [_P] * 5 + [_I] * 8 + [_F, _I, _P]),
    "llmc_rope_append_decode_strided": (_I, [_P] * 10 + [_I] + [_P] * 5 + [_I] * 8
                                        + [_F, _I, ctypes.c_longlong, ctypes.c_longlong, _I,
                                           _P]),
    "llmc_decode_gemm_workspace_bytes": (_SZ, [_I, _I, _I]),
    "llmc_decode_gemm": (_I, [_P, _P, _P, _P, _SZ, _P, _I, _I, _I, _P, _P]),
    "llmc_add_rmsnorm": (_I, [_P, _P, _P, _P, _I, _I, _F, _I, _P]),
    "llmc_swiglu": (_I, [_P, _P, _I, _I, _I, _P]),
    "llmc_argmax_workspace_bytes": (_SZ, [_I]),
    "llmc_ipc_handle_bytes": (_SZ, []),
    "llmc_ipc_alloc": (_I, [_SZ, ctypes.POINTER(ctypes.c_void_p), _P]),
    "llmc_ipc_open": (_I, [_P, ctypes.POINTER(ctypes.c_void_p)]),
    "llmc_ipc_close": (_I, [_P]),
    "llmc_ipc_free": (_I, [_P]),
    "llmc_ar_region_bytes": (_SZ, [_I, _I, _I, _I, ctypes.POINTER(_SZ)]),
    "llmc_allreduce_add_rmsnorm": (_I, [_P] * 8 + [_I] * 5 + [_F, _I, _P]),
    "llmc_argmax": (_I, [_P, _P, _I, _I, _I, _P, _P]),
    "llmc_last_error_string": (ctypes.c_char_p, []),
    "llmc_version": (ctypes.c_char_p, []),
}


class NativeLibraryError(RuntimeError):
    """The CUDA library is missing or a native call failed."""


class DeviceStatusError(RuntimeError):
    """A kernel reported an error through the device status word."""


_lib = None
_lock = threading.Lock()


def lib_path() -> str:
    return _LIB_PATH


def load() -> ctypes.CDLL:
    """Load the shared library (once).  Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                raise NativeLibraryError(
                    f"{_LIB_PATH} is missing: build it with `python -m llm_cuda_b200.build`")
            lib = ctypes.CDLL(_LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dtype]
    except KeyError:
        raise NativeLibraryError(f"unsupported dtype {dtype}") from None


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().llmc_last_error_string().decode()
        raise NativeLibraryError(f"{what} failed ({rc}): {msg}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def decode_status(word: int) -> list[str]:
    return [msg for bit, msg in STATUS_BITS.items() if word & bit]


def raise_on_status(status: torch.Tensor) -> None:
    """Synchronising check of a device status word; raises and clears it if set."""
    word = int(status.item())
    if word:
        status.zero_()
        raise DeviceStatusError("device status %#x: %s" % (word, ", ".join(decode_status(word))))
