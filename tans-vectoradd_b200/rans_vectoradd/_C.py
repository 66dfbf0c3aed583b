"""Operator surface of the reference's compiled module ``rans_vectoradd._C``
(pybind, csrc/fp8_memcpy.cu:66-78), implemented over libtans_b200's C ABI.

Same five ops, same argument meaning, same outputs and the same check
messages (raised as RuntimeError, as TORCH_CHECK does).  Differences, all
deliberate:

* launches go to torch's *current* stream of the inputs' device, under a
  device guard taken from the first tensor argument (the reference launches
  on the legacy default stream of whatever device is current);
* ``gpu_tans_decode`` builds its decode table on the device when spread and
  freqs are CUDA tensors (no host round trip); with CPU tensors it builds it
  on the host with the reference's checks, as csrc/tans_decode.cu:23-59 does;
* malformed stream metadata never makes a kernel read out of bounds; data
  errors are OR-ed into a per-device status word (``data_status``) and, with
  ``TANS_B200_CHECK=1`` in the environment, raised after every call;
* ``TANS_STREAMS_PER_BLOCK`` (csrc/vecadd.cu:245-258) is still validated, but
  the kernel geometry is chosen from the stream count and the SM count.

There is no CPU fallback: every op that the reference runs on the GPU
requires CUDA tensors and the library's sm_100a kernels.
"""
from __future__ import annotations

import ctypes
import os

import torch

from ._lib import LIB, check, lib_for_table

_L = 4096
_BLOCK = 128
_TILE_PAIRS = 8

_status_bufs: dict[int, torch.Tensor] = {}


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _status(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _status_bufs.get(idx)
    if buf is None:
        buf = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status_bufs[idx] = buf
    return buf


def data_status(device: torch.device | int | None = None, reset: bool = True) -> int:
    """Synchronise and return the OR of data-error bits (1 offsets, 2 states,
    4 table) raised by decode/fused calls on `device` since the last reset."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                       (device if isinstance(device, int) else device.index or 0))
    buf = _status(dev)
    v = int(buf.item())
    if reset:
        buf.zero_()
    return v


def _post_check(device: torch.device) -> None:
    if os.environ.get("TANS_B200_CHECK", "") not in ("", "0"):
        v = data_status(device)
        if v:
            raise RuntimeError(f"tANS data error status {v} (1 offsets, 2 states, 4 table)")


def _req(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _check_u8_cuda_contiguous(name: str, t: torch.Tensor) -> None:
    _req(t.is_cuda, f"{name} must be CUDA")
    _req(t.dtype == torch.uint8, f"{name} must be uint8")
    _req(t.is_contiguous(), f"{name} must be contiguous")


def _same_device(dev: torch.device, *ts: torch.Tensor) -> None:
    for t in ts:
        _req(t.device == dev, f"all tensors must be on {dev}; got one on {t.device}")


def _segments(n_fp8_per_stream: int, segment_pairs: int) -> int:
    """Sub-streams per stream of the split-stream format (1 when unsplit)."""
    if not segment_pairs:
        return 1
    P = n_fp8_per_stream // 2
    _req(segment_pairs > 0 and P % segment_pairs == 0,
         "segment_pairs must be a positive divisor of n_fp8_per_stream / 2")
    return P // segment_pairs


def _lib_for(n_entries: int, what: str):
    """The library for a table of n_entries: the reference's L = 4096 build,
    or the table_log 11 build (2048 entries, a labelled extra).  Other sizes
    get the reference's check message."""
    if n_entries not in (_L, _L // 2):
        raise RuntimeError(f"{what} must have {_L} entries")
    return lib_for_table(n_entries)


def _streams_per_block_from_env() -> int:
    value = os.environ.get("TANS_STREAMS_PER_BLOCK")
    if not value:
        return 8
    try:
        parsed = int(value, 10)
    except ValueError:
        raise RuntimeError("TANS_STREAMS_PER_BLOCK must be an integer") from None
    _req(parsed in (1, 2, 4, 8), "TANS_STREAMS_PER_BLOCK must be one of 1, 2, 4, or 8")
    return parsed


# ------------------------------------------------------------------ encoder

def encode_device(inp: torch.Tensor, kind: int, freqs: torch.Tensor, spread: torch.Tensor,
                  tile: int = 0, segment_pairs: int = 0):
    """Device slab encoder (csrc/encode.cu) on a contiguous CUDA uint8 input
    [K, n]: kind ENC_INPUT_FP8 (e4m3 bytes, n even; also returns the
    sign/mantissa pairs in the `tile` layout) or ENC_INPUT_SYMBOLS (pair
    symbols).  freqs/spread may live on any device.  Returns (compressed u8,
    states u16[K], offsets i32[B+1], partial u8[K], sm u8 or None), all on
    inp's device; bytes identical to the CPU encoder's.  segment_pairs > 0:
    split-stream format (K * segments sub-streams, segment-major; sm keeps
    the unsplit layout)."""
    from . import _lib
    _req(inp.is_cuda and inp.dtype == torch.uint8 and inp.dim() == 2 and inp.is_contiguous(),
         "input must be a contiguous CUDA uint8 [K, n] tensor")
    _req(freqs.dtype == torch.int32, "freqs must be int32")
    _req(spread.dtype == torch.int32, "spread must be int32")
    lib = _lib_for(spread.numel(), "spread")
    fr = freqs.detach().to("cpu").contiguous()
    sp = spread.detach().to("cpu").contiguous()
    K, n = inp.shape
    dev = inp.device
    fp8 = kind == _lib.ENC_INPUT_FP8
    P = n // 2 if fp8 else n
    S = int(segment_pairs)
    _req(S == 0 or (S > 0 and P % S == 0), "segment_pairs must divide the symbols per stream")
    chains = K * (P // S if S else 1)
    nblocks = (chains + _BLOCK - 1) // _BLOCK
    with torch.cuda.device(dev):
        wsb = ctypes.c_int64()
        check(lib.tans_b200_encode_device_workspace_bytes(K, n, kind, S, ctypes.byref(wsb)), lib)
        ws = torch.empty(wsb.value, dtype=torch.uint8, device=dev)
        states = torch.empty(chains, dtype=torch.uint16, device=dev)
        partial = torch.empty(chains, dtype=torch.uint8, device=dev)
        offsets = torch.empty(nblocks + 1, dtype=torch.int32, device=dev)
        sm = None
        if fp8:
            shape = (P // tile, K, tile) if tile > 0 and P % tile == 0 else (P, K)
            sm = torch.empty(shape, dtype=torch.uint8, device=dev)
        st = _stream(dev)
        check(lib.tans_b200_encode_device_plan(
            inp.data_ptr(), kind, K, n, tile, S, fr.data_ptr(), fr.numel(), sp.data_ptr(),
            sm.data_ptr() if sm is not None else None, states.data_ptr(), partial.data_ptr(),
            offsets.data_ptr(), ws.data_ptr(), st), lib)
        hdr = ws[:16].cpu()
        err, bad = (int(v) for v in hdr[:8].view(torch.int32))
        total = int(hdr[8:].view(torch.int64)[0])
        if err & _lib.ENC_BAD_SYMBOL:
            raise RuntimeError(f"encode: symbol {bad} occurs but has zero frequency")
        if err & _lib.ENC_TOO_LARGE:
            raise RuntimeError("encode: compressed size exceeds the int32 offsets of the format")
        comp = torch.empty(total, dtype=torch.uint8, device=dev)
        check(lib.tans_b200_encode_device_emit(kind, K, n, S, offsets.data_ptr(),
                                               ws.data_ptr(), comp.data_ptr(), st), lib)
    return comp, states, offsets, partial, sm


def tans_encode_interleaved(symbols: torch.Tensor, freqs: torch.Tensor, spread: torch.Tensor):
    """tANS encoder -> GPU-ready interleaved slab layout
    (csrc/tans_codec.cpp:69-196).  Returns (compressed u8, states u16[K],
    offsets i32[B+1], partial u8[K]): CPU tensors from CPU symbols (as the
    reference), or tensors on the symbols' device from CUDA symbols (device
    encoder, same bytes)."""
    _req(symbols.dim() == 2, "symbols must be [K, N]")
    _req(symbols.dtype == torch.uint8, "symbols must be uint8")
    _req(freqs.dtype == torch.int32, "freqs must be int32")
    _req(spread.dtype == torch.int32, "spread must be int32")
    if symbols.is_cuda:
        from ._lib import ENC_INPUT_SYMBOLS
        _req(symbols.is_contiguous(), "symbols must be contiguous")
        return encode_device(symbols, ENC_INPUT_SYMBOLS, freqs, spread)[:4]
    _req(symbols.is_contiguous() and not symbols.is_cuda, "symbols must be contiguous CPU")
    _req(freqs.is_contiguous() and not freqs.is_cuda, "freqs must be contiguous CPU")
    _req(spread.is_contiguous() and not spread.is_cuda, "spread must be contiguous CPU")
    lib = _lib_for(spread.numel(), "spread")
    K, N = symbols.shape
    h = ctypes.c_void_p()
    check(lib.tans_b200_encode(symbols.data_ptr(), K, N, freqs.data_ptr(), freqs.numel(),
                               spread.data_ptr(), 0, ctypes.byref(h)), lib)
    try:
        nbytes, nblocks = ctypes.c_int64(), ctypes.c_int64()
        check(lib.tans_b200_encoded_sizes(h, ctypes.byref(nbytes), ctypes.byref(nblocks)), lib)
        comp = torch.empty(nbytes.value, dtype=torch.uint8)
        states = torch.empty(K, dtype=torch.uint16)
        offsets = torch.empty(nblocks.value + 1, dtype=torch.int32)
        partial = torch.empty(K, dtype=torch.uint8)
        check(lib.tans_b200_encoded_export(h, comp.data_ptr(), states.data_ptr(),
                                           offsets.data_ptr(), partial.data_ptr()), lib)
    finally:
        lib.tans_b200_encoded_free(h)
    return comp, states, offsets, partial


# ------------------------------------------------------------ decode table

def build_decode_table_device(spread: torch.Tensor, freqs: torch.Tensor,
                              device: torch.device | None = None) -> torch.Tensor:
    """Reference-format decode table int32[L] on `device` (default: the
    device of spread), L = spread.numel() (4096; 2048 for table_log 11).
    Built by a kernel from CUDA inputs, on the host from CPU inputs (then
    copied)."""
    _req(spread.dtype == torch.int32, "spread must be int32")
    lib = _lib_for(spread.numel(), "spread")
    L = spread.numel()
    _req(freqs.dtype == torch.int32, "freqs must be int32")
    dev = device if device is not None else spread.device
    if spread.is_cuda and freqs.is_cuda and spread.device == dev and freqs.device == dev:
        _req(0 < freqs.numel() <= 256, "decode table alphabet must be 1..256 symbols")
        spread_c, freqs_c = spread.contiguous(), freqs.contiguous()
        with torch.cuda.device(dev):
            table = torch.empty(L, dtype=torch.int32, device=dev)
            check(lib.tans_b200_build_decode_table(spread_c.data_ptr(), freqs_c.data_ptr(),
                                                   freqs_c.numel(), table.data_ptr(),
                                                   _status(dev).data_ptr(), _stream(dev)), lib)
        return table
    sp = spread.detach().cpu().contiguous()
    fr = freqs.detach().cpu().contiguous()
    table = torch.empty(L, dtype=torch.int32)
    check(lib.tans_b200_build_decode_table_host(sp.data_ptr(), fr.data_ptr(), fr.numel(),
                                                table.data_ptr()), lib)
    return table.to(dev)


# ------------------------------------------------------------------ decode

def gpu_tans_decode(compressed: torch.Tensor, offsets: torch.Tensor, states: torch.Tensor,
                    partial_cnts: torch.Tensor, sign_mantissa: torch.Tensor,
                    spread: torch.Tensor, freqs: torch.Tensor,
                    n_fp8_per_stream: int, segment_pairs: int = 0) -> torch.Tensor:
    """GPU tANS pair decoder.  Returns [n_fp8_per_stream, n_streams] uint8
    (csrc/tans_decode.cu:159-210).  segment_pairs > 0: the inputs are in the
    split-stream format (`tans_codec.encode(..., segment_pairs=S)`)."""
    _req(compressed.is_cuda and compressed.dtype == torch.uint8 and compressed.is_contiguous(),
         "compressed must be contiguous CUDA uint8")
    _req(offsets.is_cuda and offsets.dtype == torch.int32 and offsets.is_contiguous(),
         "offsets must be contiguous CUDA int32")
    _req(states.is_cuda and states.dtype == torch.uint16 and states.is_contiguous(),
         "states must be contiguous CUDA uint16")
    _req(partial_cnts.is_cuda and partial_cnts.dtype == torch.uint8
         and partial_cnts.is_contiguous(), "partial_cnts must be contiguous CUDA uint8")
    _req(sign_mantissa.is_cuda and sign_mantissa.dtype == torch.uint8
         and sign_mantissa.is_contiguous(), "sign_mantissa must be contiguous CUDA uint8")
    N = int(n_fp8_per_stream)
    _req(N % 2 == 0, "n_fp8_per_stream must be even")
    _req(compressed.numel() % 4 == 0, "compressed length must be divisible by 4 bytes")
    S = int(segment_pairs)
    segs = _segments(N, S)
    chains = states.numel()
    _req(chains % segs == 0, "split-stream states must hold streams x segments entries")
    K = chains // segs
    n_blocks = (chains + _BLOCK - 1) // _BLOCK
    _req(offsets.numel() == n_blocks + 1, "offsets must have n_blocks + 1 entries")
    _req(partial_cnts.numel() == chains, "partial_cnts must match states")
    _req(sign_mantissa.numel() == (N // 2) * K, "sign_mantissa has the wrong shape")
    dev = compressed.device
    _same_device(dev, offsets, states, partial_cnts, sign_mantissa)
    lib = _lib_for(spread.numel(), "spread")
    with torch.cuda.device(dev):
        table = build_decode_table_device(spread, freqs, dev)
        out = torch.empty((N, K), dtype=torch.uint8, device=dev)
        args = (compressed.data_ptr(), compressed.numel(), offsets.data_ptr(), states.data_ptr(),
                partial_cnts.data_ptr(), sign_mantissa.data_ptr(), table.data_ptr(),
                out.data_ptr(), K, N)
        if S:
            check(lib.tans_b200_decode_split(*args, S, _status(dev).data_ptr(), _stream(dev)), lib)
        else:
            check(lib.tans_b200_decode(*args, _status(dev).data_ptr(), _stream(dev)), lib)
    _post_check(dev)
    return out


# ------------------------------------------------------------ memcpy / raw

def fp8_memcpy(A: torch.Tensor) -> torch.Tensor:
    """Pure HBM copy C[i] = A[i] (csrc/fp8_memcpy.cu:45-64): the practical
    bandwidth ceiling of a 1-read + 1-write SM kernel."""
    _req(A.is_cuda, "A must be CUDA")
    _req(A.dtype == torch.uint8, "A must be uint8")
    _req(A.is_contiguous(), "A must be contiguous")
    _req(A.numel() % 16 == 0, "A length must be a multiple of 16")
    with torch.cuda.device(A.device):
        C = torch.empty_like(A)
        check(LIB.tans_b200_fp8_memcpy(A.data_ptr(), C.data_ptr(), A.numel(), _stream(A.device)))
    return C


def fp8_vecadd_raw(A: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    """Uncompressed FP8 vector add C[i] = e4m3(A[i] + B[i]) with satfinite
    rounding (csrc/vecadd.cu:268-288)."""
    _check_u8_cuda_contiguous("A", A)
    _check_u8_cuda_contiguous("B", B)
    _req(A.numel() == B.numel(), "A and B must have the same length")
    _req(A.numel() % 16 == 0, "A/B length must be a multiple of 16")
    _same_device(A.device, B)
    with torch.cuda.device(A.device):
        C = torch.empty_like(A)
        check(LIB.tans_b200_fp8_vecadd_raw(A.data_ptr(), B.data_ptr(), C.data_ptr(), A.numel(),
                                           _stream(A.device)))
    return C


# ------------------------------------------------------------------ fused

def fp8_vecadd_fused_tans(a_comp: torch.Tensor, a_offsets: torch.Tensor,
                          a_states: torch.Tensor, a_partial: torch.Tensor, a_sm: torch.Tensor,
                          b_comp: torch.Tensor, b_offsets: torch.Tensor,
                          b_states: torch.Tensor, b_partial: torch.Tensor, b_sm: torch.Tensor,
                          decode_tbl: torch.Tensor, n_fp8_per_stream: int,
                          segment_pairs: int = 0) -> torch.Tensor:
    """Fused tANS decompress + FP8 vector add (csrc/vecadd.cu:290-393).
    Returns the tiled output [N/16 * K * 16] uint8.  segment_pairs > 0: both
    inputs are in the split-stream format (`tans_codec.encode(...,
    segment_pairs=S)`); the output layout is unchanged."""
    for name, t in (("a_comp", a_comp), ("a_partial", a_partial), ("a_sm", a_sm),
                    ("b_comp", b_comp), ("b_partial", b_partial), ("b_sm", b_sm)):
        _check_u8_cuda_contiguous(name, t)
    for name, t, dt, dn in (("a_offsets", a_offsets, torch.int32, "int32"),
                            ("b_offsets", b_offsets, torch.int32, "int32"),
                            ("a_states", a_states, torch.uint16, "uint16"),
                            ("b_states", b_states, torch.uint16, "uint16"),
                            ("decode_tbl", decode_tbl, torch.int32, "int32")):
        _req(t.is_cuda and t.dtype == dt and t.is_contiguous(),
             f"{name} must be contiguous CUDA {dn}")
    _req(a_states.numel() == b_states.numel(), "A/B stream counts must match")
    _req(a_partial.numel() == a_states.numel() and b_partial.numel() == b_states.numel(),
         "partial-count tensors must match state tensors")
    _req(a_comp.numel() % 4 == 0 and b_comp.numel() % 4 == 0,
         "compressed tensors must have byte lengths divisible by 4")
    lib = _lib_for(decode_tbl.numel(), "decode_tbl")
    N = int(n_fp8_per_stream)
    _req(N % (2 * _TILE_PAIRS) == 0, f"n_fp8_per_stream must be divisible by {2 * _TILE_PAIRS}")
    S = int(segment_pairs)
    segs = _segments(N, S)
    _req(a_states.numel() % segs == 0, "split-stream states must hold streams x segments entries")
    K = a_states.numel() // segs
    n_enc_blocks = (K * segs + _BLOCK - 1) // _BLOCK
    _req(a_offsets.numel() == n_enc_blocks + 1 and b_offsets.numel() == n_enc_blocks + 1,
         "offset tensors must have n_encoder_blocks + 1 entries")
    n_tiles = (N // 2) // _TILE_PAIRS
    expected_sm = n_tiles * K * _TILE_PAIRS
    _req(a_sm.numel() == expected_sm and b_sm.numel() == expected_sm,
         "sign/mantissa tensors have the wrong tiled size")
    dev = a_comp.device
    _same_device(dev, a_offsets, a_states, a_partial, a_sm, b_comp, b_offsets, b_states,
                 b_partial, b_sm, decode_tbl)
    _streams_per_block_from_env()
    with torch.cuda.device(dev):
        out = torch.empty(n_tiles * K * _TILE_PAIRS * 2, dtype=torch.uint8, device=dev)
        args = (a_comp.data_ptr(), a_comp.numel(), a_offsets.data_ptr(), a_states.data_ptr(),
                a_partial.data_ptr(), a_sm.data_ptr(),
                b_comp.data_ptr(), b_comp.numel(), b_offsets.data_ptr(), b_states.data_ptr(),
                b_partial.data_ptr(), b_sm.data_ptr(), decode_tbl.data_ptr(), out.data_ptr(), K, N)
        if S:
            check(lib.tans_b200_fp8_vecadd_fused_split(*args, S, _status(dev).data_ptr(),
                                                        _stream(dev)), lib)
        else:
            check(lib.tans_b200_fp8_vecadd_fused(*args, _status(dev).data_ptr(), _stream(dev)), lib)
    _post_check(dev)
    return out


_host_ws: dict[tuple[int, int], torch.Tensor] = {}


def fp8_vecadd_fused_tans_host(a_comp: torch.Tensor, a_offsets: torch.Tensor,
                               a_states: torch.Tensor, a_partial: torch.Tensor,
                               a_sm: torch.Tensor, b_comp: torch.Tensor,
                               b_offsets: torch.Tensor, b_states: torch.Tensor,
                               b_partial: torch.Tensor, b_sm: torch.Tensor,
                               decode_tbl: torch.Tensor, n_fp8_per_stream: int,
                               out: torch.Tensor | None = None,
                               device: torch.device | int | None = None,
                               chunk_streams: int = 0) -> torch.Tensor:
    """fp8_vecadd_fused_tans on HOST tensors (no reference counterpart): the
    inputs are copied to `device` in chunks of encoder blocks and the tiled
    output [N/16 * K * 16] is copied back into `out` (a host tensor; pinned
    if allocated here), with copies and kernels pipelined over three CUDA
    streams.  Asynchronous with respect to the host, like a non-blocking
    copy: synchronise the device's current stream before reading `out`.
    Page-locked inputs are needed for the copies to overlap."""
    ts = (a_comp, a_offsets, a_states, a_partial, a_sm, b_comp, b_offsets, b_states, b_partial,
          b_sm, decode_tbl)
    for t in ts:
        _req(not t.is_cuda and t.is_contiguous(), "host inputs must be contiguous CPU tensors")
    _req(a_states.dtype == torch.uint16 and b_states.dtype == torch.uint16, "states must be uint16")
    _req(a_offsets.dtype == torch.int32 and b_offsets.dtype == torch.int32, "offsets must be int32")
    _req(decode_tbl.dtype == torch.int32 and decode_tbl.numel() in (_L, _L // 2),
         f"decode_tbl must be {_L} int32 entries")
    lib = _lib_for(decode_tbl.numel(), "decode_tbl")
    N = int(n_fp8_per_stream)
    _req(N % (2 * _TILE_PAIRS) == 0, f"n_fp8_per_stream must be divisible by {2 * _TILE_PAIRS}")
    K = a_states.numel()
    _req(b_states.numel() == K, "A/B stream counts must match")
    nb = (K + _BLOCK - 1) // _BLOCK
    _req(a_offsets.numel() == nb + 1 and b_offsets.numel() == nb + 1,
         "offset tensors must have n_encoder_blocks + 1 entries")
    _req(a_partial.numel() == K and b_partial.numel() == K, "partial-count tensors must match")
    _req(a_sm.numel() == K * N // 2 and b_sm.numel() == K * N // 2,
         "sign/mantissa tensors have the wrong tiled size")
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                       (device if isinstance(device, int) else device.index or 0))
    if out is None:
        out = torch.empty(K * N, dtype=torch.uint8, pin_memory=True)
    _req(not out.is_cuda and out.is_contiguous() and out.numel() == K * N and
         out.dtype == torch.uint8, "out must be a contiguous CPU uint8 tensor of K*N bytes")
    with torch.cuda.device(dev):
        need = ctypes.c_int64()
        check(lib.tans_b200_fp8_vecadd_fused_host_workspace_bytes(
            K, N, a_comp.numel(), b_comp.numel(), ctypes.byref(need)), lib)
        key = (dev.index, need.value)
        ws = _host_ws.get(key)
        if ws is None:
            _host_ws.clear()
            ws = torch.empty(need.value, dtype=torch.uint8, device=dev)
            _host_ws[key] = ws
        check(lib.tans_b200_fp8_vecadd_fused_host(
            a_comp.data_ptr(), a_comp.numel(), a_offsets.data_ptr(), a_states.data_ptr(),
            a_partial.data_ptr(), a_sm.data_ptr(),
            b_comp.data_ptr(), b_comp.numel(), b_offsets.data_ptr(), b_states.data_ptr(),
            b_partial.data_ptr(), b_sm.data_ptr(), decode_tbl.data_ptr(), out.data_ptr(), K, N,
            int(chunk_streams), ws.data_ptr(), ws.numel(), _status(dev).data_ptr(), _stream(dev)),
            lib)
    return out


__all__ = ["tans_encode_interleaved", "gpu_tans_decode", "fp8_memcpy", "fp8_vecadd_raw",
           "fp8_vecadd_fused_tans", "fp8_vecadd_fused_tans_host", "build_decode_table_device",
           "data_status", "encode_device"]
