"""Bindings of the C ABI in include/gqa_fa_b200.h.

Two in-tree libraries (``make`` in the package directory, or
``__graft_entry__.build()``): ``libgqa_fa_b200.so``, the kernels behind the C
ABI, bound here with ctypes for every entry point; and ``libgqa_fa_ops.so``,
torch operators ``torch.ops.gqafa.fwd`` / ``torch.ops.gqafa.bwd`` over the
same ABI, which the autograd function's hot path calls (no per-call Python
argument marshalling). There is no CPU or Triton fallback: if a library is
missing, loading it raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get(
    "GQAFA_LIB", os.path.join(os.path.dirname(_HERE), "libgqa_fa_b200.so")
)

GQAFA_DTYPE_FP16 = 0
GQAFA_DTYPE_BF16 = 1
GQAFA_OK = 0
GQAFA_ERR_INVALID = 1
GQAFA_ERR_UNSUPPORTED = 2
GQAFA_ERR_CUDA = 3

# Every symbol include/gqa_fa_b200.h declares.
EXPORTED_SYMBOLS = (
    "gqafa_fwd",
    "gqafa_fwd_kv",
    "gqafa_bwd",
    "gqafa_bwd_stage",
    "gqafa_bwd_noalloc",
    "gqafa_bwd_ws",
    "gqafa_bwd_ws_stage",
    "gqafa_bwd_partial",
    "gqafa_bwd_workspace_size",
    "gqafa_fwd_rows",
    "gqafa_bwd_stage_rows",
    "gqafa_supported",
    "gqafa_last_error",
    "gqafa_device_status",
    "gqafa_version",
    "gqafa_set_wait_counters",
    "gqafa_set_test_waits",
)

OPS_PATH = os.path.join(os.path.dirname(LIB_PATH), "libgqa_fa_ops.so")

_lock = threading.Lock()
_lib = None
_ops = None

_P = ctypes.c_void_p
_S = ctypes.POINTER(ctypes.c_longlong)
_I = ctypes.c_int
_F = ctypes.c_float


class GQAFAError(RuntimeError):
    """A CUDA-side failure reported by the library."""


def load():
    """Load the shared library once and declare the argument types."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"gemma_triton_flash_attn: CUDA library not found at {LIB_PATH}. "
                "Build it with `make -C gemma-triton-flash-attn_b200` (nvcc, sm_100a). "
                "There is no CPU fallback."
            )
        lib = ctypes.CDLL(LIB_PATH)
        lib.gqafa_fwd.argtypes = [_P, _S, _P, _S, _P, _S, _P, _S, _P, _I, _I, _I, _I, _I, _F, _I, _I, _I, _P]
        lib.gqafa_fwd.restype = _I
        lib.gqafa_fwd_kv.argtypes = [_P, _S, _P, _S, _P, _S, _P, _S, _P, _I, _I, _I, _I, _I, _I, _F, _I, _I, _I, _P]
        lib.gqafa_fwd_kv.restype = _I
        lib.gqafa_bwd.argtypes = (
            [_P, _S, _P, _S, _P, _S, _P, _S, _P, _S, _P, _P, _S, _P, _S, _P, _S, _P]
            + [_I, _I, _I, _I, _I, _F, _I, _I, _I, _P]
        )
        lib.gqafa_bwd.restype = _I
        lib.gqafa_bwd_stage.argtypes = [_I] + lib.gqafa_bwd.argtypes
        lib.gqafa_bwd_stage.restype = _I
        lib.gqafa_fwd_rows.argtypes = lib.gqafa_fwd.argtypes + [_I, _I]
        lib.gqafa_fwd_rows.restype = _I
        lib.gqafa_bwd_stage_rows.argtypes = [_I] + lib.gqafa_bwd.argtypes + [_I, _I]
        lib.gqafa_bwd_stage_rows.restype = _I
        lib.gqafa_bwd_noalloc.argtypes = (
            [_P, _S, _P, _S, _P, _S, _P, _S, _P, _S, _P, _P, _S, _P, _S, _P, _S]
            + [_I, _I, _I, _I, _I, _F, _I, _I, _I, _P]
        )
        lib.gqafa_bwd_noalloc.restype = _I
        _L = ctypes.c_longlong
        lib.gqafa_bwd_ws.argtypes = lib.gqafa_bwd.argtypes + [_P, _L]
        lib.gqafa_bwd_ws.restype = _I
        lib.gqafa_bwd_ws_stage.argtypes = [_I] + lib.gqafa_bwd.argtypes + [_P, _L]
        lib.gqafa_bwd_ws_stage.restype = _I
        lib.gqafa_bwd_partial.argtypes = lib.gqafa_bwd.argtypes + [_P, _L]
        lib.gqafa_bwd_partial.restype = _I
        lib.gqafa_bwd_workspace_size.argtypes = [_I] * 7
        lib.gqafa_bwd_workspace_size.restype = _L
        lib.gqafa_supported.argtypes = [_I, _I]
        lib.gqafa_supported.restype = _I
        lib.gqafa_last_error.argtypes = []
        lib.gqafa_last_error.restype = ctypes.c_char_p
        lib.gqafa_device_status.argtypes = [_I, _I]
        lib.gqafa_device_status.restype = _I
        lib.gqafa_set_wait_counters.argtypes = [_P]
        lib.gqafa_set_wait_counters.restype = _I
        lib.gqafa_set_test_waits.argtypes = [ctypes.c_longlong, _I]
        lib.gqafa_set_test_waits.restype = _I
        lib.gqafa_version.argtypes = []
        lib.gqafa_version.restype = ctypes.c_char_p
        _lib = lib
        return lib


def ops():
    """torch.ops.gqafa, loading libgqa_fa_ops.so on first use."""
    global _ops
    with _lock:
        if _ops is None:
            if not os.path.exists(OPS_PATH):
                raise ImportError(
                    f"gemma_triton_flash_attn: torch operator library not found at {OPS_PATH}. "
                    "Build it with `make -C gemma-triton-flash-attn_b200`. There is no CPU fallback."
                )
            import torch

            torch.ops.load_library(OPS_PATH)
            _ops = torch.ops.gqafa
    return _ops


def strides_arg(strides):
    """A 4-element stride array (elements) for the ABI."""
    arr = (ctypes.c_longlong * 4)(*[int(s) for s in strides])
    return arr


def check(rc: int) -> None:
    """Turn a non-zero return code into the exception the reference would raise."""
    if rc == GQAFA_OK:
        return
    msg = load().gqafa_last_error().decode(errors="replace")
    if rc == GQAFA_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    if rc == GQAFA_ERR_INVALID:
        raise ValueError(msg)
    raise GQAFAError(msg)


def device_status(device: int, reset: bool = True) -> int:
    """Synchronise `device` and return the kernels' status word (0 = healthy)."""
    return int(load().gqafa_device_status(int(device), 1 if reset else 0))


def version() -> str:
    return load().gqafa_version().decode()
