"""ctypes binding of the C-ABI library ``libqwen3_b200_attn.so`` (include/qwen3_b200_attn.h).

The library is built in-tree by ``build.py`` (nvcc, sm_100a).  Loading it is
the only way into the kernels: there is no CPU or eager-PyTorch fallback, so a
missing library raises immediately.
"""

from __future__ import annotations

import ctypes
import os
import threading

LIB_NAME = "libqwen3_b200_attn.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

B200_OK = 0
B200_ERR_INVALID_ARGUMENT = -1
B200_ERR_UNSUPPORTED = -2
B200_ERR_ALIGNMENT = -3
B200_ERR_WORKSPACE = -4
B200_ERR_CUDA = -5
B200_ERR_TENSOR_MAP = -6

DEV_BAD_ROW = 0x1
DEV_BAD_PAGE = 0x2
DEV_BAD_SLOT = 0x4
DEV_SEQ_OVERFLOW = 0x8
DEV_TIMEOUT = 0x10
DEV_BAD_PARAM = 0x20

DEV_STATUS_NAMES = {
    DEV_BAD_ROW: "row id outside the block table",
    DEV_BAD_PAGE: "block-table entry outside the pool",
    DEV_BAD_SLOT: "slot_mapping entry outside the pool",
    DEV_SEQ_OVERFLOW: "sequence position past the block table",
    DEV_TIMEOUT: "pipeline wait timed out",
    DEV_BAD_PARAM: "per-row parameter outside its range (clamped)",
}

# Every symbol include/qwen3_b200_attn.h declares, with its ctypes signature.
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_F = ctypes.c_float
_SZ = ctypes.c_size_t

SIGNATURES = {
    "b200_status_string": (ctypes.c_char_p, [_I]),
    "b200_abi_version": (_I, []),
    "b200_last_cuda_error_string": (ctypes.c_char_p, []),
    "b200_device_sm_count": (_I, []),
    "b200_selftest_bounded_wait": (_I, [_P, _P, ctypes.c_uint64, _P]),
    "b200_kv_scatter_rows": (_I, [_P, _P, _I64, _I64, _I64, _I64, _I64, _I64,
                                  _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64,
                                  _P, _P, _I64, _P,
                                  _I, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P]),
    "b200_kv_scatter_slots": (_I, [_P, _P, _I64, _I64, _I64, _I64,
                                   _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64,
                                   _P, _I, _I, _I, _I, _I, _I, _I, _P, _P]),
    "b200_kv_scatter_span": (_I, [_P, _P, _I64, _I64, _I64, _I64,
                                  _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64,
                                  _P, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P]),
    "b200_paged_decode_workspace_size": (_SZ, [_I, _I, _I, _I]),
    "b200_paged_decode_default_split": (_I, [_I, _I, _I]),
    "b200_paged_decode": (_I, [_P, _I64, _I64, _P, _P, _I64, _I64, _I64,
                               _P, _I64, _P, _P, _P, _I64, _I64,
                               _I, _I, _I, _I, _I, _I, _I, _I, _F, _I,
                               _P, _SZ, _P, _P]),
    "b200_paged_decode_kv_write": (_I, [_P, _I64, _I64, _P, _I64, _I64, _P, _I64, _I64,
                                        _P, _P, _I64, _I64, _I64,
                                        _P, _I64, _P, _P, _P, _I64, _I64,
                                        _I, _I, _I, _I, _I, _I, _I, _I, _F, _I,
                                        _P, _SZ, _P, _P]),
    "b200_paged_decode_noalloc": (_I, [_P, _I64, _I64, _P, _P, _I64, _I64, _I64,
                                       _P, _I64, _P, _P, _P, _I64, _I64,
                                       _I, _I, _I, _I, _I, _I, _I, _I, _F, _I, _P, _P]),
    "b200_varlen_prefill": (_I, [_P, _I64, _I64, _P, _I64, _I64, _P, _I64, _I64,
                                 _P, _I64, _I64, _P, _P, _I, _I, _I, _I, _I, _I,
                                 _F, _I, _P, _P, _P]),
    "b200_sample_workspace_size": (_SZ, [_I, _I, _I]),
    "b200_sample_tokens": (_I, [_P, _I, _I64, _I, _I, _P, _P, _P, _F, _I, _F, ctypes.c_uint64,
                                _I, _P, _SZ, _P, _P, _P]),
    "b200_paged_prefill": (_I, [_P, _I64, _I64, _P, _P, _I64, _I64, _I64, _P, _I64, _P, _P,
                                _P, _P, _I64, _I64, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I,
                                _F, _P, _P, _P]),
    "b200_qk_norm_rope_kv_write": (_I, [_P, _I64, _I64, _I64, _P, _I64, _I64, _I64,
                                        _P, _I64, _I64, _I64, _P, _P, _F, _P, _P, _I64, _I64,
                                        _P, _I64, _I64, _I64, _P, _I64, _I64, _I64,
                                        _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64,
                                        _P, _P, _I64, _P,
                                        _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P]),
}

_lib = None
_lock = threading.Lock()


class NativeLibraryMissing(RuntimeError):
    pass


def load() -> ctypes.CDLL:
    """Load the C-ABI library (once) and declare its signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise NativeLibraryMissing(
                f"{LIB_NAME} is not built (expected at {LIB_PATH}); build it with "
                "`python -m qwen3_engine_from_scratch_b200.build` -- there is no fallback path")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def status_string(code: int) -> str:
    return load().b200_status_string(int(code)).decode()


def check(code: int, what: str) -> None:
    """Map a non-zero C status to RuntimeError (the reference raises on bad input too)."""
    if code != B200_OK:
        detail = ""
        if code == B200_ERR_CUDA:
            detail = f": {load().b200_last_cuda_error_string().decode()}"
        raise RuntimeError(f"{what} failed: {status_string(code)}{detail} (status {code})")


def describe_dev_status(bits: int) -> str:
    return ", ".join(msg for b, msg in DEV_STATUS_NAMES.items() if bits & b) or "ok"
