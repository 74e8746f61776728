"""ctypes binding of libmi_paged.so (the C ABI declared in include/mi_paged.h).

The library is loaded lazily on first use and must exist: there is no fallback of any kind.  A
missing library raises ``RuntimeError`` naming the build command.  Every wrapper checks the
return code: ``MI_ERR_INVALID`` becomes ``ValueError`` (an argument the host rejected, like the
reference's shape checks), the other codes become ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from mini_infra_b200.build import LIB_PATH

MI_F32, MI_BF16, MI_F16 = 0, 1, 2
MI_OK, MI_ERR_INVALID, MI_ERR_CUDA, MI_ERR_UNSUPPORTED = 0, -1, -2, -3
MI_STATUS_BAD_BLOCK, MI_STATUS_BAD_SLOT, MI_STATUS_TIMEOUT, MI_STATUS_BAD_LENGTH, MI_STATUS_BAD_INDEX = 1, 2, 4, 8, 16

# Every symbol of include/*.h with its ctypes signature (restype, argtypes).
_P = ctypes.c_void_p
_I64P = ctypes.POINTER(ctypes.c_int64)
_I = ctypes.c_int
_L = ctypes.c_int64
SIGNATURES: dict[str, tuple] = {
    "mi_version": (_I, []),
    "mi_last_error": (ctypes.c_char_p, []),
    "mi_read_status": (_I, [ctypes.POINTER(ctypes.c_uint), _I, _P]),
    "mi_kv_scatter": (_I, [_P, _P, _I64P, _I64P, _L, _L, _P, _P, _P, _L, _P, _P, _L, _I, _I, _I, _I, _P]),
    "mi_kv_store_chunks": (_I, [_P, _P, _I64P, _I64P, _L, _L, _P, _P, _P, _L, _P, _P, _L, _I, _I, _I, _I, _P]),
    "mi_kv_gather_blocks": (_I, [_P, _P, _L, _L, _P, _L, _I, _I, _I, _I, _P]),
    "mi_paged_decode_workspace_size": (ctypes.c_size_t, [_L, _I, _I, _I, _L, _I, _I]),
    "mi_paged_decode": (
        _I,
        [_P, _I64P, _P, _P, _I64P, _P, _P, _P, _L, _I, _I, _I, _P, _L, _L, _P, _L, _I, ctypes.c_float, _P, _L, _P,
         ctypes.c_size_t, _I, _P],
    ),
    "mi_paged_decode_static_scratch": (
        _I,
        [_P, _I64P, _P, _P, _I64P, _P, _P, _P, _L, _I, _I, _I, _P, _L, _L, _P, _L, _I, ctypes.c_float, _P, _L, _I, _P],
    ),
    "mi_paged_decode_exchange": (
        _I,
        [_P, _I64P, _P, _P, _I64P, _P, _P, _P, _L, _I, _I, _I, _P, _L, _L, _P, _L, _I, ctypes.c_float, _P, _L, _P, _P,
         _I, _I, _L, _P, ctypes.c_size_t, _I, _P],
    ),
    "mi_peer_handle": (_I, [_P, _P, _I64P]),
    "mi_peer_open": (_I, [_P, _L, ctypes.POINTER(ctypes.c_void_p)]),
    "mi_peer_close": (_I, [_P, _L]),
    "mi_paged_prefill_workspace_size": (ctypes.c_size_t, [_L, _L, _I, _I, _I, _L, _I, _I]),
    "mi_paged_prefill": (
        _I,
        [_P, _I64P, _P, _P, _I64P, _P, _P, _L, _I, _I, _I, _P, _L, _P, _P, _L, _L, _I, ctypes.c_float, _P, _P,
         ctypes.c_size_t, _I, _P],
    ),
    "mi_decode_rows": (_I, [_P, _L, _P, _L, _P, _L, _L, _P, _L, _L, _I, _P]),
    # include/mi_layers.h
    "mi_rmsnorm": (_I, [_P, _L, _P, _L, _P, _L, _P, _P, _L, _L, _I, ctypes.c_float, _I, _P]),
    "mi_qk_norm_rope": (
        _I,
        [_P, _L, _P, _L, _P, _L, _P, _P, _P, _P, _L, _L, _I, _I, _I, ctypes.c_float, _P, _P, _P, _P, _P, _P, _L, _I,
         _P],
    ),
    "mi_silu_mul": (_I, [_P, _P, _L, _P, _L, _L, _L, _I, _P]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def library_path() -> Path:
    return LIB_PATH


def load() -> ctypes.CDLL:
    """Load (once) and return the library with typed entry points."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"libmi_paged.so not found at {LIB_PATH}; build it with `python -m mini_infra_b200.build` "
                    "(this package has no CPU or PyTorch fallback)"
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = lib
    return _lib


def last_error() -> str:
    return load().mi_last_error().decode("utf-8", "replace")


def check(rc: int, what: str) -> None:
    if rc == MI_OK:
        return
    msg = f"{what}: {last_error()}"
    if rc == MI_ERR_INVALID:
        raise ValueError(msg)
    raise RuntimeError(msg)


def i64_array(values) -> ctypes.Array:
    return (ctypes.c_int64 * len(values))(*[int(v) for v in values])
