"""ctypes binding of the C-ABI library (include/agentserve_b200.h).

The library is the only compute path: if it is missing, every op raises
NativeLibraryError — there is no Python or CPU fallback.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libagentserve_b200.so"

AS_OK = 0
AS_ERR_INVALID_ARG = 1
AS_ERR_UNSUPPORTED = 2
AS_ERR_CUDA = 3
AS_ERR_WORKSPACE = 4

AS_DTYPE_F32 = 0
AS_DTYPE_F16 = 1
AS_DTYPE_BF16 = 2

AS_LAYOUT_HEAD_MAJOR = 0
AS_LAYOUT_DIM_MAJOR = 1

AS_DECODE_NOALLOC_SCRATCH_BYTES = 8 << 20

AS_KERNEL_DECODE_ATTENTION = 1
AS_KERNEL_PREFILL_ATTENTION = 2

# Every exported entry point with its C signature (restype, argtypes).
_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_F32 = ctypes.c_float
_SZ = ctypes.c_size_t
SIGNATURES = {
    "as_version": (ctypes.c_int, []),
    "as_last_error": (ctypes.c_char_p, []),
    "as_device_status": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_int), _P]),
    "as_pack_decode": (ctypes.c_int, [_P, _I64, _P, _P, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P]),
    "as_pack_prefill": (ctypes.c_int, [_P, _I64, _P, _P, _P, _I32, _I32, _I32, _I32, _P, _P, _P,
                                       _P, _P, _P]),
    "as_rope_reshape_and_cache": (ctypes.c_int, [_P, _I64, _P, _I64, _P, _I64, _P, _P, _P, _I32,
                                                 _P, _P, _I64, _P, _I32, _I32, _I32, _I32, _I32,
                                                 _P]),
    "as_paged_decode_workspace_size": (_SZ, [_I32, _I32, _I32, _I32, _I32, _I32]),
    "as_paged_decode_attention": (ctypes.c_int, [_P, _P, _I64, _P, _P, _P, _I64, _P, _I32, _I32,
                                                 _I32, _I32, _I32, _I32, _I32, _F32, _I32, _P,
                                                 _SZ, _I32, _I32, _P]),
    "as_paged_decode_attention_noalloc": (ctypes.c_int, [_P, _P, _I64, _P, _P, _P, _I64, _P,
                                                         _I32, _I32, _I32, _I32, _I32, _I32,
                                                         _I32, _F32, _I32, _I32, _I32, _P]),
    "as_varlen_prefill_attention": (ctypes.c_int, [_P, _P, _I64, _P, _P, _P, _I64, _P, _P, _I32,
                                                   _I32, _I32, _I32, _I32, _I32, _I32, _I32,
                                                   _I32, _F32, _I32, _P]),
    "as_varlen_prefill_attention_ws": (ctypes.c_int, [_P, _P, _I64, _P, _P, _P, _I64, _P, _P,
                                                      _I32, _I32, _I32, _I32, _I32, _I32, _I32,
                                                      _I32, _I32, _F32, _I32, _I32, _P, _SZ,
                                                      _P]),
    "as_varlen_prefill_workspace_size": (_SZ, [_I32, _I32, _I32, _I32, _I32, _I32, _I32, _I32]),
    "as_linear_small_m": (ctypes.c_int, [_P, _I64, _P, _I64, _P, _I32, _I32, _I32, _I32, _P]),
    "as_linear_small_m_swiglu": (ctypes.c_int, [_P, _I64, _P, _I64, _P, _I32, _I32, _I32, _I32,
                                                _P]),
    "as_greedy_workspace_size": (_SZ, [_I32]),
    "as_greedy_argmax": (ctypes.c_int, [_P, _P, _I64, _I32, _I32, _I32, _P, _SZ, _P]),
    "as_rmsnorm": (ctypes.c_int, [_P, _P, _P, _I64, _I32, _F32, _I32, _P]),
    "as_add_rmsnorm": (ctypes.c_int, [_P, _P, _P, _P, _I64, _I32, _F32, _I32, _P]),
    "as_silu_mul": (ctypes.c_int, [_P, _P, _I64, _I32, _I32, _P]),
    "as_block_copy": (ctypes.c_int, [_P, _P, _P, _P, _I32, _I64, _I32, _I64, _I64, _I32, _I32,
                                     _P]),
    "as_rope_paged_decode_attention": (ctypes.c_int, [_P, _P, _I64, _P, _I64, _P, _I64, _P, _P,
                                                      _P, _I32, _P, _P, _P, _I64, _P, _I32, _I32,
                                                      _I32, _I32, _I32, _I32, _I32, _F32, _I32,
                                                      _P, _SZ, _I32, _I32, _P]),
    "as_set_wait_limit_ns": (ctypes.c_uint64, [ctypes.c_uint64]),
    "as_debug_starve_next_launch": (ctypes.c_int, [ctypes.c_int]),
}


class NativeLibraryError(RuntimeError):
    """The sm_100a library is missing or failed to load."""


class KernelError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


_lib = None
_lock = threading.Lock()


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load the library once (no compute call is made)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise NativeLibraryError(
                f"{p} not found: build it with `python -m agentserve_b200.build` "
                "(there is no CPU fallback)")
        try:
            lib = ctypes.CDLL(str(p))
        except OSError as e:  # pragma: no cover - depends on the environment
            raise NativeLibraryError(f"cannot load {p}: {e}") from e
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def last_error() -> str:
    msg = load().as_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str) -> None:
    if rc == AS_OK:
        return
    msg = last_error() or what
    if rc in (AS_ERR_INVALID_ARG, AS_ERR_WORKSPACE):
        raise ValueError(msg)
    raise KernelError(rc, msg)
