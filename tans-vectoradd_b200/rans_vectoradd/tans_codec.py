"""tANS codec front-end for FP8 pair-alphabet streams.

Public surface of the reference's rans_vectoradd/tans_codec.py (constants
:24-27, quantize_freqs :30-46, build_spread :49-60, build_decode_table
:63-87, encode :90-143) with the same arguments, outputs and bytes.

An e4m3 byte splits into a 4-bit exponent, entropy-coded in pairs with tANS
(pair symbol = exp(2i) << 4 | exp(2i+1), alphabet 256), and a sign+mantissa
nibble stored uncompressed (sm(2i) | sm(2i+1) << 4 per pair).  The heavy
lifting (nibble split, tiling, slab encode) runs in C++ with OpenMP inside
libtans_b200; table construction is vectorised numpy here.

Table size: L = 4096 (table_log 12) is the reference's and the parity path.
`encode(..., table_log=11)` is a labelled extra with a 2048-entry table
(pair frequencies quantised to 2048, the same spread rule with its own
stride); every op infers L from the spread / decode-table size and runs the
library build for it.

Wire format: each stream is a sequence of uint32 slabs filled LSB-first;
the final partial slab stays LSB-aligned and `partial_cnts` gives its bit
count; 128-stream blocks pad every stream to the block's slab count G_b with
streams top-aligned (lower slab indices zero).
"""
from __future__ import annotations

import numpy as np
import torch

from . import _C
from ._lib import LIB, check

L = 4096
M = L
SIGMA = (L >> 1) + (L >> 3) + 3  # hash-walk stride (odd, so it visits every slot)
BLOCK_STREAMS = 128
TABLE_LOGS = (12, 11)  # 12: the reference's L; 11: the labelled extra


def _table_size(n: int) -> int:
    if n not in [1 << t for t in TABLE_LOGS]:
        raise AssertionError(f"freqs must sum to {L}")
    return n


def quantize_freqs(probs: np.ndarray, target: int = M) -> np.ndarray:
    """Integer frequencies summing to `target`: round-half-even of
    probs*target, at least 1 for every p > 0, then one unit at a time to the
    symbol whose rounding error is largest (lowest index on ties) until the
    sum is exact."""
    p = np.asarray(probs, dtype=np.float64)
    zero = p == 0
    f = np.maximum(np.round(p * target).astype(np.int64), 1)
    f[zero] = 0
    while True:
        short = target - int(f.sum())
        if short == 0:
            break
        if short > 0:
            score = p * target - f
            score[zero] = -np.inf
            f[int(np.argmax(score))] += 1
        else:
            score = f - p * target
            score[~zero & (f <= 1)] = -np.inf
            f[int(np.argmax(score))] -= 1
    return f.astype(np.int32)


def build_spread(freqs: np.ndarray) -> np.ndarray:
    """Slot -> symbol map: the j-th placed symbol (symbols in order, symbol s
    repeated f_s times) goes to slot (j * SIGMA) mod L, L = sum of freqs
    (4096; 2048 for table_log 11, stride (L >> 1) + (L >> 3) + 3 likewise)."""
    f = np.asarray(freqs, dtype=np.int64)
    Lt = _table_size(int(f.sum()))
    sigma = (Lt >> 1) + (Lt >> 3) + 3
    if (f < 0).any():
        # quantize_freqs can drive a zero-probability symbol to -1 when it has
        # to remove units (as the reference's does); the reference's spread
        # then trips its slot assertion
        raise AssertionError("freqs must be non-negative")
    spread = np.full(Lt, -1, dtype=np.int32)
    spread[(np.arange(Lt, dtype=np.int64) * sigma) % Lt] = np.repeat(
        np.arange(f.size, dtype=np.int32), f)
    return spread


def build_decode_table(spread: np.ndarray, freqs: np.ndarray) -> torch.Tensor:
    """[L] int32 decode table, entry = sym | nb << 8 | base << 16 (L =
    spread size: 4096, or 2048 for table_log 11).

    For slot j holding symbol s with rank r among the slots of s (ascending
    slot order): x' = f_s + r, nb lifts x' into [L, 2L), base = x' << nb.  A
    decoder at state x = L + j reads nb bits and moves to base | bits."""
    sp = np.asarray(spread, dtype=np.int64)
    fr = np.asarray(freqs, dtype=np.int64)
    Lt = sp.size
    if Lt not in [1 << t for t in TABLE_LOGS] or sp.min() < 0 or sp.max() >= fr.size:
        raise AssertionError("spread does not match freqs")
    counts = np.bincount(sp, minlength=fr.size)
    first = np.concatenate(([0], np.cumsum(counts)[:-1]))
    order = np.argsort(sp, kind="stable")
    rank = np.empty(Lt, dtype=np.int64)
    rank[order] = np.arange(Lt, dtype=np.int64) - np.repeat(first, counts)
    xp = fr[sp] + rank
    if (xp <= 0).any():
        raise AssertionError("spread does not match freqs")
    nb = (Lt.bit_length() - 1) - (np.frexp(xp.astype(np.float64))[1] - 1)
    base = xp << nb
    if not ((base >= Lt) & (base < 2 * Lt)).all():
        raise AssertionError("spread does not match freqs")
    table = ((sp & 0xFF) | (nb << 8) | (base << 16)).astype(np.uint32)
    return torch.from_numpy(table.view(np.int32))


def pair_freqs_from_exponents(exp_freqs, table_log: int = 12) -> np.ndarray:
    """Pair-symbol frequencies from 16 exponent weights: the outer product of
    the normalised nibble probabilities (float32, as the reference computes
    them), quantised to sum to M = 2^table_log (4096 in the reference)."""
    if table_log not in TABLE_LOGS:
        raise AssertionError(f"table_log must be one of {TABLE_LOGS}")
    probs = torch.as_tensor(exp_freqs).float().numpy()
    probs = probs / probs.sum()
    return quantize_freqs((probs[:, None] * probs[None, :]).flatten(), target=1 << table_log)


def split_fp8(fp8_bytes: torch.Tensor, tile: int = 0, want_hist: bool = False):
    """(pair_syms u8[K, N/2], sm_packed, exp_hist int64[16] or None) of an
    e4m3 byte matrix [K, N]; sm_packed is [N/2/tile, K, tile] for tile > 0,
    else [N/2, K]."""
    src = fp8_bytes.detach().to("cpu").contiguous()
    K, N = src.shape
    P = N // 2
    syms = torch.empty((K, P), dtype=torch.uint8)
    if tile > 0:
        sm = torch.empty((P // tile, K, tile), dtype=torch.uint8)
    else:
        sm = torch.empty((P, K), dtype=torch.uint8)
    hist = torch.zeros(16, dtype=torch.int64) if want_hist else None
    check(LIB.tans_b200_split_fp8(src.data_ptr(), K, N, tile, syms.data_ptr(), sm.data_ptr(),
                                  hist.data_ptr() if hist is not None else None, 0))
    return syms, sm, hist


def encode(
    fp8_bytes: torch.Tensor,
    exp_freqs: torch.Tensor,
    tile: int = 0,
    segment_pairs: int = 0,
    table_log: int = 12,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
           torch.Tensor, torch.Tensor, torch.Tensor]:
    """tANS encode FP8 bytes [K, N] (pair alphabet).

    If tile > 0, sm_packed is returned in tiled layout [n_tiles, K, tile] for
    fused vecadd, otherwise [N/2, K] for standalone decode.

    Returns compressed [bytes], final_states [K], block_offsets
    [n_blocks+1], partial_cnts [K] (uint8), sm_packed, pair_freqs, spread.
    CPU input encodes on the host (as the reference); CUDA input encodes on
    its device (split + slab encode kernels) and the first five outputs stay
    there.  Bytes are identical either way.

    segment_pairs = S > 0 (a format extension, not in the reference): every
    stream is cut into N/2/S sub-streams of S pair symbols, encoded as
    independent streams in segment-major order (sub-stream j*K + k is pairs
    [jS, (j+1)S) of stream k) — the reference encoder's bytes for the
    pair-symbol matrix rearranged that way; sm_packed keeps the unsplit
    layout.  Long streams then decode as N/2/S times as many chains
    (gpu_tans_decode / fp8_vecadd_fused_tans with segment_pairs=S).

    table_log = 11 (a labelled extra; the reference has only 12): pair
    frequencies sum to 2048 and spread has 2048 entries; the decode ops
    recognise that size and use the 2048-entry library build.
    """
    assert fp8_bytes.dim() == 2 and fp8_bytes.dtype == torch.uint8
    K, N = fp8_bytes.shape
    assert N % 2 == 0
    if tile > 0:
        n_pairs = N // 2
        assert n_pairs % tile == 0, f"n_pairs={n_pairs} not divisible by tile={tile}"
    if segment_pairs:
        assert segment_pairs > 0 and (N // 2) % segment_pairs == 0, \
            f"segment_pairs={segment_pairs} must divide n_pairs={N // 2}"
    pair_freqs = pair_freqs_from_exponents(exp_freqs, table_log)
    spread = build_spread(pair_freqs)
    pair_freqs_t = torch.from_numpy(pair_freqs)
    spread_t = torch.from_numpy(spread)
    if fp8_bytes.is_cuda:
        # device encoder: split and slab encode on the GPU, outputs stay there
        from ._lib import ENC_INPUT_FP8
        compressed, states, offsets, partial_cnts, sm_packed = _C.encode_device(
            fp8_bytes.contiguous(), ENC_INPUT_FP8, pair_freqs_t, spread_t, tile, segment_pairs)
        return (compressed, states, offsets, partial_cnts, sm_packed, pair_freqs_t, spread_t)
    pair_syms, sm_packed, _ = split_fp8(fp8_bytes, tile)
    if segment_pairs and segment_pairs != N // 2:
        S = segment_pairs
        pair_syms = pair_syms.view(K, N // 2 // S, S).transpose(0, 1).reshape(-1, S).contiguous()
    compressed, states, offsets, partial_cnts = _C.tans_encode_interleaved(
        pair_syms, pair_freqs_t, spread_t)
    return (compressed, states, offsets, partial_cnts, sm_packed, pair_freqs_t, spread_t)
