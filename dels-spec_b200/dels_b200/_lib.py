"""ctypes binding of the C ABI declared in ``include/dels_b200.h``.

The shared library is the in-tree ``libdels_b200.so`` built by :mod:`dels_b200.build`.
There is no fallback: if the library is missing or cannot be loaded, every operation
raises, so a run can never silently score tokens on another code path.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libdels_b200.so"

DELS_OK = 0
DELS_ERR_INVALID_ARG = -1
DELS_ERR_ALIGNMENT = -2
DELS_ERR_WORKSPACE = -3
DELS_ERR_CUDA = -4
DELS_ERR_UNSUPPORTED = -5
DELS_ERR_DEVICE_TIMEOUT = -6

DELS_ACT_IDENTITY = 0
DELS_ACT_SILU = 1
DELS_FLAG_KEYS_READY = 1
DELS_WS_HEADER_BYTES = 256
DELS_NOALLOC_SCRATCH_BYTES = 12 * 1024 * 1024

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_U32 = ctypes.c_uint32
_SZ = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/dels_b200.h one to one.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "dels_version": (_I, []),
    "dels_status_string": (ctypes.c_char_p, [_I]),
    "dels_last_error": (ctypes.c_char_p, []),
    "dels_init": (_I, [_I]),
    "dels_sm_count": (_I, [_I]),
    "dels_rank_workspace_bytes": (_SZ, [_I, _I, _I]),
    "dels_rank_project_bf16": (
        _I,
        [_P, _I64, _P, _I64, _I, _I, _I, _I, _P, _I, _P, _P, _P, _P, _P, _SZ, _P],
    ),
    "dels_fused_argmax_bf16": (
        _I,
        [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _P, _I, _P, _I, _P, _I, _I, _I, _I64, _U32, _P, _P, _P, _P,
         _SZ, _P],
    ),
    "dels_fused_argmax_base_bf16": (
        _I,
        [_P, _I64, _P, _I64, _P, _I64, _P, _P, _I, _P, _I, _P, _I, _I, _I64, _U32, _P, _P, _P, _P, _SZ, _P],
    ),
    "dels_score_workspace_bytes": (_SZ, [_I, _I, _I]),
    "dels_draft_score_bf16": (
        _I,
        [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _P, _P, _I, _P, _I, _P, _I, _I, _I, _I64, _I, _P, _P, _P, _P,
         _SZ, _P],
    ),
    "dels_score_f32_workspace_bytes": (_SZ, [_I, _I, _I]),
    "dels_draft_score_f32": (
        _I,
        [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _P, _P, _I, _P, _I, _I, _I, _I, _I64, _P, _P, _P, _P, _SZ,
         _P],
    ),
    "dels_keys_init": (_I, [_P, _I, _P, _P]),
    "dels_keys_decode": (_I, [_P, _I, _P, _P, _P, _P]),
    "dels_accept_offsets": (_I, [_P, _I64, _P, _I64, _I, _I, _I, _P, _P, _P]),
    "dels_pack_rows_bf16": (_I, [_P, _I64, _I64, _I, _I, _I, _P, _P, _P, _I64, _P, _P]),
    "dels_rnn_workspace_bytes": (_SZ, [_I, _I, _I, _I]),
    "dels_rnn_rank_states_bf16": (
        _I,
        [_P, _I64, _P, _I64, _P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _SZ, _P],
    ),
    "dels_gru_step_bf16": (_I, [_P, _I64, _I, _P, _I64, _P, _P, _P, _P, _I, _I, _I, _P, _P]),
    "dels_fused_argmax_base_gru_bf16": (_I, [_P, _I64, _P, _I64, _P, _I64, _P, _P, _I, _I, _I, _I, _U32, _P, _P,
                                             _P, _SZ, _P, _P, _P, _I, _P, _P]),
    "dels_gru_correction_mid_bf16": (_I, [_P, _I64, _I, _P, _I64, _P, _I64, _P, _P, _I, _I, _I, _P, _I64, _P, _I64,
                                          _I, _P, _P, _P, _P, _P]),
    "dels_gru_rank_gemv_bf16": (_I, [_P, _I64, _I, _P, _I64, _P, _I64, _P, _P, _I, _I, _I, _P, _I64, _P, _I, _I, _P,
                                     _P, _P, _P, _P]),
    "dels_gru_gates_bf16": (_I, [_P, _I64, _I, _P, _I64, _P, _I64, _P, _P, _I, _I, _I, _P, _P]),
    "dels_rank_gemv_bf16": (_I, [_P, _I64, _P, _I64, _P, _I, _I, _I, _I, _P, _I, _P, _P, _P, _P, _P, _P]),
    "dels_gather_scaled_rows_bf16": (_I, [_P, _I64, _I, _P, _I64, _P, _I, _I, _I, _I, _P, _P, _P, _P]),
    "dels_gru_step_tc_workspace_bytes": (_SZ, [_I, _I]),
    "dels_gru_step_tc_bf16": (_I, [_P, _I64, _I, _P, _I64, _P, _P, _P, _P, _I, _I, _I, _P, _SZ, _P]),
    "dels_linear_workspace_bytes": (_SZ, [_I, _I, _I]),
    "dels_correction_mid_tc_workspace_bytes": (_SZ, [_I, _I, _I]),
    "dels_linear_bf16": (_I, [_P, _I64, _P, _I64, _P, _I, _I, _I, _P, _I64, _P, _SZ, _P]),
    "dels_correction_mid_bf16": (_I, [_P, _I64, _P, _I64, _P, _I64, _I, _I, _I, _P, _P, _P, _P, _P]),
    "dels_correction_mid_tc_bf16": (_I, [_P, _I64, _P, _I64, _P, _I64, _I, _I, _I, _P, _P, _P, _P, _SZ, _P]),
    "dels_selftest_bounded_wait": (_I, [_P, _P, ctypes.c_double, _P]),
    "dels_draft_score_bf16_noalloc": (
        _I,
        [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _P, _P, _I, _P, _I, _P, _I, _I, _I, _I64, _I, _P, _P, _P, _P],
    ),
    "dels_noalloc_status": (_I, [_P, _I, _P]),
    "dels_selftest_bounded_wait_noalloc": (_I, [_P, ctypes.c_double, _P]),
}


class DelsError(RuntimeError):
    """A dels_* entry point returned a non-zero status."""

    def __init__(self, fn: str, status: int, message: str):
        self.fn = fn
        self.status = status
        super().__init__(f"{fn} failed with status {status}: {message}")


class DelsArgumentError(DelsError, ValueError):
    """Invalid shapes, strides, alignment or workspace (the reference raises ValueError)."""


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load ``libdels_b200.so`` (once) and declare every exported signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with dels_b200.build.build() "
                "(or __graft_entry__.build()); there is no non-CUDA fallback"
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    return list(SIGNATURES)


def call(name: str, *args) -> int:
    """Call an int-returning entry point and raise on a non-zero status."""
    lib = load()
    status = getattr(lib, name)(*args)
    if status != DELS_OK:
        msg = (lib.dels_last_error() or b"").decode(errors="replace")
        if status in (DELS_ERR_INVALID_ARG, DELS_ERR_ALIGNMENT, DELS_ERR_WORKSPACE):
            raise DelsArgumentError(name, status, msg)
        raise DelsError(name, status, msg)
    return status


def query(name: str, *args):
    """Call an entry point that returns a value (sizes, counts) rather than a status."""
    return getattr(load(), name)(*args)
