"""ctypes binding of ``libiris_b200.so`` (the C ABI in include/iris_b200.h).

There is no fallback: if the library is missing or cannot be loaded the
import fails with the reason, so a GPU run can never silently take another
path.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libiris_b200.so")

IRIS_OK = 0
STATUS_NAMES = {1: "EINVAL", 2: "EUNSUPPORTED", 3: "EALIGN", 4: "ECUDA", 5: "EWORKSPACE"}

ERR_SLOT_RANGE = 0x1
ERR_POS_NEGATIVE = 0x2
ERR_POS_RANGE = 0x4
ERR_DUP_SLOT = 0x8
ERR_SEQ_LEN = 0x10
ERR_BLOCK_TABLE = 0x20
ERR_PAGE_ID = 0x40
ERR_PIPELINE_TIMEOUT = 0x80

DECODE_OUT_FP16 = 0
DECODE_OUT_LSE = 1

DECODE_NOALLOC_SCRATCH_BYTES = 32 << 20  # IRIS_DECODE_NOALLOC_SCRATCH_BYTES
APPEND_INLINE_CHECK_TOKENS = 128  # IRIS_APPEND_INLINE_CHECK_TOKENS

_c_i32, _c_i64, _c_sz, _c_p, _c_f = ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_float

# name -> (restype, argtypes); must match include/iris_b200.h
SIGNATURES = {
    "iris_b200_version": (ctypes.c_int, []),
    "iris_b200_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "iris_b200_last_cuda_error": (ctypes.c_char_p, []),
    "iris_b200_append_check_workspace_bytes": (_c_sz, [_c_i64, _c_i32]),
    "iris_b200_append_check": (ctypes.c_int, [_c_p, _c_p, _c_i64, _c_i64, _c_i64, _c_i32, _c_p, _c_sz, _c_p, _c_p]),
    "iris_b200_rope_int4_paged_append": (
        ctypes.c_int,
        [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_i64, _c_i32, _c_i32, _c_i64, _c_i64, _c_i32,
         _c_p, _c_p]),
    "iris_b200_decode_workspace_bytes": (_c_sz, [_c_i32, _c_i32, _c_i32, _c_i32, _c_i32]),
    "iris_b200_int4_paged_decode": (
        ctypes.c_int,
        [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_i64, _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32,
         _c_i64, _c_i32, _c_i32, _c_f, _c_p, _c_sz, _c_p, _c_p]),
    "iris_b200_int4_paged_decode_noalloc": (
        ctypes.c_int,
        [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_i64, _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32,
         _c_i64, _c_i32, _c_i32, _c_f, _c_p, _c_p]),
    "iris_b200_merge_lse_partials": (ctypes.c_int, [_c_p, _c_p, _c_i32, _c_i64, _c_i32, _c_p, _c_p]),
    "iris_b200_merge_lse_packed": (ctypes.c_int, [_c_p, _c_i32, _c_i64, _c_i32, _c_p, _c_p]),
    "iris_b200_selftest_bounded_wait": (ctypes.c_int, [_c_p, _c_i64, _c_p]),
    "iris_b200_selftest_quantizer_sweep": (ctypes.c_int, [_c_i32, _c_i32, _c_p, _c_p]),
    "iris_b200_int4_quantize_pack": (ctypes.c_int, [_c_p, _c_p, _c_p, _c_i64, _c_i32, _c_p]),
    "iris_b200_rope_fp16_paged_append": (
        ctypes.c_int,
        [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_i64, _c_i32, _c_i32, _c_i32, _c_i64, _c_i64, _c_i32, _c_p,
         _c_p]),
    "iris_b200_fp16_decode_workspace_bytes": (_c_sz, [_c_i32, _c_i32, _c_i32, _c_i32, _c_i32]),
    "iris_b200_fp16_paged_decode": (
        ctypes.c_int,
        [_c_p, _c_p, _c_p, _c_p, _c_i64, _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i64, _c_i32,
         _c_i32, _c_f, _c_p, _c_sz, _c_p, _c_p]),
    "iris_b200_xchg_buffer_bytes": (_c_sz, [_c_i64, _c_i32]),
    "iris_b200_xchg_alloc": (ctypes.c_int, [_c_sz, ctypes.POINTER(_c_p)]),
    "iris_b200_xchg_free": (ctypes.c_int, [_c_p]),
    "iris_b200_ipc_export": (ctypes.c_int, [_c_p, _c_p]),
    "iris_b200_ipc_open": (ctypes.c_int, [_c_p, ctypes.POINTER(_c_p)]),
    "iris_b200_ipc_close": (ctypes.c_int, [_c_p]),
    "iris_b200_xchg_merge": (ctypes.c_int, [ctypes.POINTER(_c_p), _c_i32, _c_i32, _c_i64, _c_i32, _c_p, _c_p, _c_p,
                                            _c_p, _c_i64, _c_p]),
}

IPC_HANDLE_BYTES = 64  # IRIS_IPC_HANDLE_BYTES
XCHG_HEADER_BYTES = 256  # IRIS_XCHG_HEADER_BYTES


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"iris_kernel: {LIB_PATH} is missing; build it with `python iris-kernel_b200/build.py` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def check_status(status: int, what: str) -> None:
    if status != IRIS_OK:
        msg = lib.iris_b200_status_string(status).decode()
        detail = lib.iris_b200_last_cuda_error().decode() if status == 4 else ""
        raise RuntimeError(f"{what} failed: {msg} ({STATUS_NAMES.get(status, status)}) {detail}".rstrip())
