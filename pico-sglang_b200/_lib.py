"""ctypes binding of libpgb.so (the C ABI in include/pgb.h).

The library is loaded from this package directory only; there is no
fallback implementation. A missing library raises at first use with the
command that builds it.
"""

from __future__ import annotations

import ctypes
import threading
from ctypes import POINTER, c_char_p, c_float, c_int, c_longlong, c_size_t, c_uint8, c_uint64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libpgb.so"

PGB_OK = 0
PGB_ERR_INVALID = 1
PGB_ERR_CUDA = 2
PGB_ERR_TIMEOUT = 3
PGB_ERR_UNSUPPORTED = 4
PGB_ERR_STATE = 5

PGB_F16 = 0
PGB_BF16 = 1
PGB_F32 = 2
PGB_I32 = 3
PGB_I64 = 4
PGB_OP_SUM = 0
PGB_XCHG_AUTO = 0
PGB_XCHG_ONESHOT = 1
PGB_XCHG_TWOSHOT = 2
PGB_XCHG_BARRIER = 3
PGB_XCHG_NVLS = 4
UID_BYTES = 128
MAX_RANKS = 8

_ERR_NAMES = {
    PGB_ERR_INVALID: "invalid argument",
    PGB_ERR_CUDA: "CUDA error",
    PGB_ERR_TIMEOUT: "device wait timed out",
    PGB_ERR_UNSUPPORTED: "unsupported",
    PGB_ERR_STATE: "bad state",
}


class PGBError(RuntimeError):
    """A libpgb call returned a non-zero status (see include/pgb.h)."""

    def __init__(self, code: int, where: str, message: str):
        self.code = code
        super().__init__(f"{where}: {_ERR_NAMES.get(code, code)}: {message}")


class PGBTimeout(PGBError):
    """A bounded device-side wait on a peer or on the pipeline ran out."""


# Signatures: name -> (restype, argtypes). Mirrors include/pgb.h.
_SIGS: dict[str, tuple[object, list[object]]] = {
    "pgb_last_error": (c_char_p, []),
    "pgb_version": (c_int, []),
    "pgb_create_uid": (c_int, [POINTER(c_uint8)]),
    "pgb_comm_create": (c_int, [c_int, c_int, c_size_t, POINTER(c_uint8), c_int, POINTER(c_void_p)]),
    "pgb_comm_handle_size": (c_int, []),
    "pgb_comm_export_handle": (c_int, [c_void_p, c_void_p, POINTER(c_uint8)]),
    "pgb_comm_open_peers": (c_int, [c_void_p, POINTER(c_uint8)]),
    "pgb_comm_destroy": (c_int, [c_void_p]),
    "pgb_comm_set_timeout_ns": (c_int, [c_void_p, c_uint64]),
    "pgb_comm_get_status": (c_int, [c_void_p, POINTER(c_int), c_int]),
    "pgb_comm_set_one_rank_path": (c_int, [c_void_p, c_int]),
    "pgb_comm_set_exchange_mode": (c_int, [c_void_p, c_int]),
    "pgb_comm_nvls_supported": (c_int, [c_void_p, POINTER(c_int)]),
    "pgb_comm_nvls_create": (c_int, [c_void_p, POINTER(c_int)]),
    "pgb_comm_nvls_add": (c_int, [c_void_p, c_int]),
    "pgb_comm_nvls_bind": (c_int, [c_void_p]),
    "pgb_comm_get_buffer": (c_int, [c_void_p, POINTER(c_void_p)]),
    "pgb_all_reduce": (c_int, [c_void_p, c_void_p, c_size_t, c_int, c_int, c_void_p]),
    "pgb_all_gather": (c_int, [c_void_p, c_void_p, c_void_p, c_size_t, c_int, c_void_p]),
    "pgb_col_gemm_workspace_size": (c_size_t, [c_int, c_int, c_int]),
    "pgb_col_gemm": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p],
    ),
    "pgb_col_gemm_noalloc": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p],
    ),
    "pgb_col_gemm_noalloc_status": (c_int, [POINTER(c_int), c_int]),
    "pgb_gate_up_silu_workspace_size": (c_size_t, [c_int, c_int, c_int, c_int]),
    "pgb_gate_up_silu": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p],
    ),
    "pgb_silu_and_mul": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "pgb_qkv_rope_store_workspace_size": (c_size_t, [c_int, c_int, c_int, c_int, c_int, c_int]),
    "pgb_qkv_rope_store": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_int,
         c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_longlong, c_int, c_void_p, c_size_t, c_void_p],
    ),
    "pgb_rope_store": (
        c_int,
        [c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p,
         c_void_p, c_void_p, c_longlong, c_int, c_void_p, c_void_p],
    ),
    "pgb_row_gemm_allreduce_addnorm": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_int, c_int,
         c_int, c_int, c_void_p],
    ),
    "pgb_fused_add_rmsnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_float, c_int, c_int, c_int, c_void_p]),
    "pgb_rmsnorm": (c_int, [c_void_p, c_void_p, c_float, c_void_p, c_int, c_int, c_int, c_void_p]),
    "pgb_check_work_plan": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, c_int]),
    "pgb_launch_features": (c_int, []),
    "pgb_describe_plan": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, c_char_p, c_size_t]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load libpgb.so once and attach argument/return types."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python {LIB_PATH.parent / 'build.py'}`"
            )
        lib = ctypes.CDLL(str(LIB_PATH), mode=ctypes.RTLD_LOCAL)
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def declared_symbols() -> list[str]:
    return list(_SIGS)


def check(code: int, where: str) -> None:
    """Raise PGBError (PGBTimeout for PGB_ERR_TIMEOUT) when code != 0."""
    if code == PGB_OK:
        return
    msg = load().pgb_last_error()
    text = msg.decode(errors="replace") if msg else ""
    cls = PGBTimeout if code == PGB_ERR_TIMEOUT else PGBError
    raise cls(code, where, text)


def call(name: str, *args):
    """Call a status-returning entry point and raise on failure."""
    check(getattr(load(), name)(*args), name)
