"""ctypes binding of libtans_b200.so (C ABI: include/tans_b200.h).

The library is loaded from this package directory.  There is no fallback:
if it is missing or does not load, importing rans_vectoradd raises.  A second
build with a 2048-entry table (table_log 11, a labelled extra beside the
reference's L = 4096) is loaded on first use by `lib_for_table(2048)`.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libtans_b200.so")
LIB_PATH_L11 = os.path.join(_HERE, "libtans_b200_l11.so")

OK = 0
DATA_BAD_OFFSETS = 1
DATA_BAD_STATE = 2
DATA_BAD_TABLE = 4
ENC_INPUT_FP8 = 0
ENC_INPUT_SYMBOLS = 1
ENC_TOO_LARGE = 1
ENC_BAD_SYMBOL = 2


def _load(path: str = LIB_PATH, table_size: int = 4096) -> ctypes.CDLL:
    if not os.path.exists(path):
        raise ImportError(
            f"{path} is missing: build it with `python tans-vectoradd_b200/build.py` "
            "(rans_vectoradd has no CPU fallback)")
    lib = ctypes.CDLL(path)
    p, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    sig = {
        "tans_b200_last_error": (ctypes.c_char_p, []),
        "tans_b200_version": (ctypes.c_char_p, []),
        "tans_b200_table_size": (i32, []),
        "tans_b200_build_decode_table_host": (i32, [p, p, i64, p]),
        "tans_b200_encode": (i32, [p, i64, i64, p, i64, p, i32, ctypes.POINTER(p)]),
        "tans_b200_encoded_sizes": (i32, [p, ctypes.POINTER(i64), ctypes.POINTER(i64)]),
        "tans_b200_encoded_export": (i32, [p, p, p, p, p]),
        "tans_b200_encoded_free": (None, [p]),
        "tans_b200_split_fp8": (i32, [p, i64, i64, i64, p, p, p, i32]),
        "tans_b200_sm_count": (i32, [ctypes.POINTER(i32)]),
        "tans_b200_fp8_memcpy": (i32, [p, p, i64, p]),
        "tans_b200_fp8_vecadd_raw": (i32, [p, p, p, i64, p]),
        "tans_b200_build_decode_table": (i32, [p, p, i64, p, p, p]),
        "tans_b200_decode": (i32, [p, i64, p, p, p, p, p, p, i64, i64, p, p]),
        "tans_b200_fp8_vecadd_fused": (i32, [p, i64, p, p, p, p, p, i64, p, p, p, p, p, p,
                                             i64, i64, p, p]),
        "tans_b200_decode_noalloc": (i32, [p, i64, p, p, p, p, p, p, i64, p, i64, i64, p, p]),
        "tans_b200_gemv": (i32, [p, i64, p, p, p, p, p, p, p, p, p, i64, i64, i64, i64, p, p]),
        "tans_b200_gemv_gather": (i32, [p, i64, p, p, p, p, p, p, p, p, i64, i64, i64, i64, p, p,
                                        p]),
        "tans_b200_gemv_weight_dense": (i32, [p, i64, p, p, p, p, p, p, i64, i64, i64, p, p]),
        "tans_b200_gemv_raw": (i32, [p, p, p, p, p, i64, i64, i64, i64, p]),
        "tans_b200_scale_rows_bf16": (i32, [p, p, p, i64, i64, p]),
        "tans_b200_gemm_tc": (i32, [p, i64, p, p, p, p, p, p, p, p, i64, i64, i64, i64, p, p]),
        "tans_b200_fp8_vecadd_fused_range": (i32, [p, i64, p, p, p, p, p, i64, p, p, p, p, p, p,
                                                   i64, i64, i64, i64, p, p]),
        "tans_b200_fp8_vecadd_fused_host_workspace_bytes": (i32, [i64, i64, i64, i64,
                                                                  ctypes.POINTER(i64)]),
        "tans_b200_fp8_vecadd_fused_host": (i32, [p, i64, p, p, p, p, p, i64, p, p, p, p, p, p,
                                                  i64, i64, i64, p, i64, p, p]),
        "tans_b200_encode_device_workspace_bytes": (i32, [i64, i64, i32, i64,
                                                          ctypes.POINTER(i64)]),
        "tans_b200_encode_device_plan": (i32, [p, i32, i64, i64, i64, i64, p, i64, p, p, p, p,
                                               p, p, p]),
        "tans_b200_encode_device_emit": (i32, [i32, i64, i64, i64, p, p, p, p]),
        "tans_b200_fp8_vecadd_fused_split": (i32, [p, i64, p, p, p, p, p, i64, p, p, p, p, p, p,
                                                   i64, i64, i64, p, p]),
        "tans_b200_decode_split": (i32, [p, i64, p, p, p, p, p, p, i64, i64, i64, p, p]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.tans_b200_table_size() != table_size:
        raise ImportError(f"{path} was built for L = {lib.tans_b200_table_size()}, "
                          f"expected {table_size}")
    return lib


LIB = _load()
_LIB_L11: ctypes.CDLL | None = None


def lib_for_table(size: int) -> ctypes.CDLL:
    """The library built for a decode table of `size` entries: 4096 (the
    reference's L, the parity path) or 2048 (table_log 11)."""
    global _LIB_L11
    if size == 4096:
        return LIB
    if size == 2048:
        if _LIB_L11 is None:
            try:
                _LIB_L11 = _load(LIB_PATH_L11, 2048)
            except ImportError as e:
                raise RuntimeError(str(e)) from None
        return _LIB_L11
    raise RuntimeError(f"no library build for a {size}-entry table (4096, or 2048 for table_log 11)")


def check(rc: int, lib: ctypes.CDLL | None = None) -> None:
    """Raise RuntimeError (what TORCH_CHECK raises) for a nonzero status;
    `lib` is the library that made the call (default: the L = 4096 one)."""
    if rc != OK:
        msg = (lib or LIB).tans_b200_last_error().decode(errors="replace")
        raise RuntimeError(msg or f"libtans_b200 error {rc}")


def version() -> str:
    return LIB.tans_b200_version().decode()
