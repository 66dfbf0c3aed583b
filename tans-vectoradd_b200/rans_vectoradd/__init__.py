"""rans_vectoradd — B200-native (sm_100a) tANS FP8 decode path.

Drop-in for the reference package of the same name
(doublewordai/tans-vectoradd, rans_vectoradd/__init__.py:1-18): the same
exports, backed by hand-written sm_100a kernels in libtans_b200.so.
"""
from rans_vectoradd._C import (
    fp8_memcpy,
    fp8_vecadd_fused_tans,
    fp8_vecadd_raw,
    gpu_tans_decode,
)
from rans_vectoradd.data import QWEN3_14B_FP8_EXP, random_fp8_bytes
from . import tans_codec

__all__ = [
    "QWEN3_14B_FP8_EXP",
    "fp8_memcpy",
    "fp8_vecadd_fused_tans",
    "fp8_vecadd_raw",
    "gpu_tans_decode",
    "random_fp8_bytes",
    "tans_codec",
]
