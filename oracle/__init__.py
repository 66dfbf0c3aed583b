"""CPU oracle for the tANS FP8 hot path — TEST INFRASTRUCTURE ONLY.

ctypes wrapper over ``oracle/liboracle.so`` (built from ``tans_oracle.c`` by
``oracle/Makefile``), plus a loader for the reference's own extension built
from its sources into ``oracle/_ref`` by ``oracle/build_ref.sh``.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` leg of
``bench.py`` may import this package.  The product never does.

Function map (reference file:line each one restates):
  fp8_add_table / vecadd_raw   csrc/vecadd.cu:27-35, 41-73
  build_decode_table           rans_vectoradd/tans_codec.py:63-87
  encode                       csrc/tans_codec.cpp:22-60, 69-196
  decode                       csrc/tans_decode.cu:65-155
  vecadd_fused                 csrc/vecadd.cu:84-154, 156-243
  quantize_freqs / build_spread / encode_front
                               rans_vectoradd/tans_codec.py:24-27, 30-60, 90-143
                               (numpy, so that a caller can encode with the
                               reference's own compiled encoder without the
                               product package)
"""
from __future__ import annotations

import ctypes
import glob
import importlib.util
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None


def build() -> None:
    """Compile liboracle.so (and nothing else)."""
    subprocess.run(["make", "-s", "-C", HERE, "liboracle.so"], check=True)


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = ctypes.CDLL(path)
        p = ctypes.c_void_p
        i64 = ctypes.c_int64
        L.oracle_e4m3_to_double.restype = ctypes.c_double
        L.oracle_e4m3_to_double.argtypes = [ctypes.c_uint8]
        L.oracle_e4m3_from_double.restype = ctypes.c_uint8
        L.oracle_e4m3_from_double.argtypes = [ctypes.c_double]
        L.oracle_fp8_add.restype = ctypes.c_uint8
        L.oracle_fp8_add.argtypes = [ctypes.c_uint8, ctypes.c_uint8]
        L.oracle_fp8_add_table.argtypes = [p]
        L.oracle_vecadd_raw.argtypes = [p, p, p, i64]
        L.oracle_build_decode_table.restype = ctypes.c_int
        L.oracle_build_decode_table.argtypes = [p, p, ctypes.c_int, p]
        L.oracle_encode.restype = i64
        L.oracle_encode.argtypes = [p, i64, i64, p, ctypes.c_int, p, p, p, p, p]
        L.oracle_decode.restype = ctypes.c_int
        L.oracle_decode.argtypes = [p, i64, p, p, p, p, p, i64, i64, p]
        L.oracle_vecadd_fused.restype = ctypes.c_int
        L.oracle_vecadd_fused.argtypes = [p, i64, p, p, p, p, p, i64, p, p, p, p, p, i64, i64, p]
        L.oracle_decode_l.restype = ctypes.c_int
        L.oracle_decode_l.argtypes = [p, i64, p, p, p, p, p, i64, i64, p, i64]
        L.oracle_vecadd_fused_l.restype = ctypes.c_int
        L.oracle_vecadd_fused_l.argtypes = [p, i64, p, p, p, p, p, i64, p, p, p, p, p, i64, i64, p,
                                            i64]
        L.oracle_num_threads.restype = ctypes.c_int
        L.oracle_set_num_threads.restype = None
        L.oracle_set_num_threads.argtypes = [ctypes.c_int]
        _LIB = L
    return _LIB


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data


def _np(x, dtype) -> np.ndarray:
    """Host numpy copy of a tensor/array, reinterpreted (same width) or cast to dtype."""
    if hasattr(x, "detach"):  # torch tensor
        x = x.detach().cpu().contiguous().numpy()
    x = np.asarray(x)
    if x.dtype != dtype:
        x = x.view(dtype) if x.dtype.itemsize == np.dtype(dtype).itemsize else x.astype(dtype)
    return np.ascontiguousarray(x)


def num_threads() -> int:
    return int(lib().oracle_num_threads())


def set_num_threads(n: int) -> None:
    """OpenMP threads of the oracle's parallel loops (n > 0)."""
    lib().oracle_set_num_threads(int(n))


def fp8_add(a: int, b: int) -> int:
    return int(lib().oracle_fp8_add(a, b))


def fp8_add_table() -> np.ndarray:
    """uint8[256, 256]: satfinite e4m3(a + b) for every byte pair."""
    out = np.empty((256, 256), np.uint8)
    lib().oracle_fp8_add_table(_p(out))
    return out


def vecadd_raw(a, b) -> np.ndarray:
    a = _np(a, np.uint8).ravel()
    b = _np(b, np.uint8).ravel()
    c = np.empty_like(a)
    lib().oracle_vecadd_raw(_p(a), _p(b), _p(c), a.size)
    return c


def build_decode_table(spread, freqs) -> np.ndarray:
    spread = _np(spread, np.int32)
    freqs = _np(freqs, np.int32)
    out = np.empty(4096, np.int32)
    rc = lib().oracle_build_decode_table(_p(spread), _p(freqs), freqs.size, _p(out))
    if rc != 0:
        raise ValueError("oracle: inconsistent spread/freqs")
    return out


def encode(symbols, freqs, spread):
    """symbols uint8[K, N] -> (compressed u8, states u16[K], offsets i32[B+1], partial u8[K])."""
    sym = _np(symbols, np.uint8)
    K, N = sym.shape
    freqs = _np(freqs, np.int32)
    spread = _np(spread, np.int32)
    L = lib()
    B = (K + 127) // 128
    offsets = np.empty(B + 1, np.int32)
    total = L.oracle_encode(_p(sym), K, N, _p(freqs), freqs.size, _p(spread), None, None,
                            _p(offsets), None)
    if total < 0:
        raise ValueError("oracle: encode failed")
    comp = np.empty(total, np.uint8)
    states = np.empty(K, np.uint16)
    partial = np.empty(K, np.uint8)
    L.oracle_encode(_p(sym), K, N, _p(freqs), freqs.size, _p(spread), _p(comp), _p(states),
                    _p(offsets), _p(partial))
    return comp, states, offsets, partial


def decode(comp, offsets, states, partial, sm, table, n_fp8_per_stream: int):
    """Returns (out uint8[N, K], ok)."""
    comp = _np(comp, np.uint8)
    offsets = _np(offsets, np.int32)
    states = _np(states, np.uint16)
    partial = _np(partial, np.uint8)
    sm = _np(sm, np.uint8)
    table = _np(table, np.int32)
    K = states.size
    N = int(n_fp8_per_stream)
    out = np.empty((N, K), np.uint8)
    # the table's size is L: 4096 (the reference's), or 2048 for the table_log 11 extra
    rc = lib().oracle_decode_l(_p(comp), comp.size, _p(offsets), _p(states), _p(partial), _p(sm),
                               _p(table), K, N, _p(out), table.size)
    return out, rc == 0


def vecadd_fused(a, b, table, n_fp8_per_stream: int):
    """a, b: (comp, offsets, states, partial, sm_tiled).  Returns (out u8[N/16*K*16], ok)."""
    ac, ao, ast, ap, asm = (_np(a[0], np.uint8), _np(a[1], np.int32), _np(a[2], np.uint16),
                            _np(a[3], np.uint8), _np(a[4], np.uint8))
    bc, bo, bst, bp, bsm = (_np(b[0], np.uint8), _np(b[1], np.int32), _np(b[2], np.uint16),
                            _np(b[3], np.uint8), _np(b[4], np.uint8))
    table = _np(table, np.int32)
    K = ast.size
    N = int(n_fp8_per_stream)
    out = np.empty(N * K, np.uint8)
    rc = lib().oracle_vecadd_fused_l(_p(ac), ac.size, _p(ao), _p(ast), _p(ap), _p(asm),
                                     _p(bc), bc.size, _p(bo), _p(bst), _p(bp), _p(bsm),
                                     _p(table), K, N, _p(out), table.size)
    return out, rc == 0


# -------------------------------------------- encode front end (numpy)

_L = 4096                            # tans_codec.py:24-25
_SIGMA = (_L >> 1) + (_L >> 3) + 3   # tans_codec.py:26


def quantize_freqs(probs) -> np.ndarray:
    """tans_codec.py:30-46: round(p * L) (half to even), floor 1 for p > 0,
    then move single units to/from the symbol with the largest rounding error
    (first index on ties) until the sum is L."""
    p = np.asarray(probs, dtype=np.float64)
    f = np.round(p * _L).astype(np.int64)
    f[(p > 0) & (f == 0)] = 1
    while int(f.sum()) != _L:
        err = p * _L - f
        if f.sum() < _L:
            err[p == 0] = -np.inf
            f[int(np.argmax(err))] += 1
        else:
            err = -err
            err[(p == 0) | (f <= 1)] = -np.inf
            f[int(np.argmax(err))] -= 1
    return f.astype(np.int32)


def build_spread(freqs) -> np.ndarray:
    """tans_codec.py:49-60: walk the slots with stride SIGMA (mod L), placing
    symbol 0 f_0 times, then symbol 1, ..."""
    spread = np.empty(_L, np.int32)
    pos = 0
    for sym, f in enumerate(np.asarray(freqs, dtype=np.int64)):
        for _ in range(int(f)):
            spread[pos] = sym
            pos = (pos + _SIGMA) % _L
    return spread


def encode_front(fp8, exp_freqs, tile: int = 8):
    """tans_codec.py:90-143 up to the slab encoder: the pair symbols
    u8[K, N/2] (exp(2i) << 4 | exp(2i+1)), the packed sign/mantissa pairs
    (sm(2i) | sm(2i+1) << 4) as [N/2/tile, K, tile] (tile > 0) or [N/2, K],
    and the pair frequencies (outer product of the float32 nibble
    probabilities) with their spread.  fp8: uint8 [K, N] e4m3 bytes."""
    b = _np(fp8, np.uint8)
    K, N = b.shape
    exp = (b >> 3) & 15
    sm = ((b >> 4) & 8) | (b & 7)
    syms = ((exp[:, 0::2] << 4) | exp[:, 1::2]).astype(np.uint8)
    pairs = (sm[:, 0::2] | (sm[:, 1::2] << 4)).astype(np.uint8)           # [K, N/2]
    if tile > 0:
        sm_out = np.ascontiguousarray(pairs.reshape(K, N // 2 // tile, tile).transpose(1, 0, 2))
    else:
        sm_out = np.ascontiguousarray(pairs.T)
    pr = np.asarray(exp_freqs, dtype=np.float64).astype(np.float32)
    pr = pr / pr.sum()
    freqs = quantize_freqs((pr[:, None] * pr[None, :]).reshape(-1))
    return syms, sm_out, freqs, build_spread(freqs)


# ------------------------------------------------------------ reference _C

def ref_ext_path() -> str | None:
    hits = sorted(glob.glob(os.path.join(HERE, "_ref", "_C*.so")))
    return hits[0] if hits else None


def load_ref_ext():
    """Import the reference's own compiled `_C` (built by build_ref.sh), or
    return None when it has not been built.  Loaded under a private parent
    name so it never shadows the product's ``rans_vectoradd._C``."""
    path = ref_ext_path()
    if path is None:
        return None
    name = "_tans_reference._C"
    if name in sys.modules:
        return sys.modules[name]
    import torch  # noqa: F401  (the extension links libtorch)
    parent = type(sys)("_tans_reference")
    parent.__path__ = []
    sys.modules.setdefault("_tans_reference", parent)
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    sys.modules[name] = mod
    return mod
