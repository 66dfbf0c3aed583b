"""On-disk container for tANS-encoded tensors, with sharded loading.

The reference declares `safetensors` as a dependency (pyproject.toml:10) but
never stores encoded data; its encoded tuple lives only in memory.  This
module writes the `tans_codec.encode` outputs (and GEMV weights) in the
safetensors file layout, so any safetensors reader can open the files:

    8 bytes   little-endian u64: header length H
    H bytes   JSON: {name: {"dtype", "shape", "data_offsets": [begin, end]},
                     "__metadata__": {str: str}}, padded with spaces so the
              data starts on a 64-byte boundary
    data      the tensors back to back (offsets relative to the data start)

Tensor names for one encoded input: compressed (U8), offsets (I32), states
(U16), partial (U8), sm (U8, [N/2, K] or [N/2/tile, K, tile]), pair_freqs
(I32), spread (I32); metadata: format, n_fp8_per_stream, tile, n_streams,
block_streams, table_log.

`load_encoded(path, rank=r, world=w)` reads only rank r's contiguous range of
whole 128-stream encoder blocks (the partition of `shard.block_range`):
its compressed byte range, states, partial counts, rebased offsets and its
columns of the sign/mantissa array, straight from a memory map into
page-locked host memory and then to the device, so a rank never touches the
other ranks' bytes.
"""
from __future__ import annotations

import json
import mmap
import os
import struct

import numpy as np
import torch

from . import shard

FORMAT = "tans-vectoradd-b200/encoded-v1"
GEMV_FORMAT = "tans-vectoradd-b200/gemv-weight-v1"
_ALIGN = 64

_DTYPES = {torch.uint8: "U8", torch.int32: "I32", torch.uint16: "U16", torch.float32: "F32",
           torch.int64: "I64"}
_NP = {"U8": np.uint8, "I32": np.int32, "U16": np.uint16, "F32": np.float32, "I64": np.int64}
_TORCH = {v: k for k, v in _DTYPES.items()}


def save(path: str, tensors: dict[str, torch.Tensor], metadata: dict[str, str] | None = None):
    """Write `tensors` (any device; copied to host) in the safetensors layout."""
    names = list(tensors)
    host = {k: tensors[k].detach().contiguous().cpu() for k in names}
    header: dict = {}
    off = 0
    for k in names:
        t = host[k]
        if t.dtype not in _DTYPES:
            raise ValueError(f"{k}: unsupported dtype {t.dtype}")
        nbytes = t.numel() * t.element_size()
        header[k] = {"dtype": _DTYPES[t.dtype], "shape": list(t.shape),
                     "data_offsets": [off, off + nbytes]}
        off += nbytes
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    blob = json.dumps(header, separators=(",", ":")).encode()
    pad = (-(8 + len(blob))) % _ALIGN
    blob += b" " * pad
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(blob)))
        f.write(blob)
        for k in names:
            t = host[k]
            if t.numel():
                f.write(t.reshape(-1).view(torch.uint8).numpy().data)
    os.replace(tmp, path)


class _File:
    """Memory-mapped container with header access and zero-copy numpy views."""

    def __init__(self, path: str):
        self._f = open(path, "rb")
        size = os.fstat(self._f.fileno()).st_size
        if size < 8:
            raise ValueError(f"{path}: not a container (too short)")
        # private (copy-on-write) mapping: the views are writable numpy arrays
        # that torch can wrap without a copy; the file itself is never written
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_COPY)
        (hlen,) = struct.unpack("<Q", self._mm[:8])
        if hlen > size - 8:
            raise ValueError(f"{path}: header length {hlen} exceeds the file")
        try:
            self.header = json.loads(bytes(self._mm[8:8 + hlen]).decode())
        except (UnicodeDecodeError, json.JSONDecodeError) as e:
            raise ValueError(f"{path}: malformed header ({e})") from None
        self.meta = self.header.pop("__metadata__", {})
        self._data = 8 + hlen
        for k, v in self.header.items():
            b, e = v["data_offsets"]
            n = int(np.prod(v["shape"], dtype=np.int64)) * np.dtype(_NP[v["dtype"]]).itemsize
            if not (0 <= b <= e <= size - self._data) or e - b != n:
                raise ValueError(f"{path}: tensor {k} has inconsistent offsets")

    def array(self, name: str) -> np.ndarray:
        v = self.header[name]
        b, _ = v["data_offsets"]
        dt = np.dtype(_NP[v["dtype"]])
        n = int(np.prod(v["shape"], dtype=np.int64))
        return np.frombuffer(self._mm, dtype=dt, count=n, offset=self._data + b).reshape(v["shape"])

    def close(self):
        self._f.close()
        try:
            self._mm.close()
        except BufferError:
            pass  # a caller still holds a view; the map closes when it is freed


def load(path: str, device=None) -> tuple[dict[str, torch.Tensor], dict[str, str]]:
    """Every tensor of the file (on `device`, default CPU) and the metadata."""
    f = _File(path)
    try:
        out = {k: _to(f.array(k), device) for k in f.header}
        return out, dict(f.meta)
    finally:
        f.close()


def _to(a: np.ndarray, device) -> torch.Tensor:
    """One copy out of the memory map (torch's multi-threaded strided copy):
    into page-locked memory for a device target, then an asynchronous
    host-to-device copy; else into a CPU tensor."""
    on_dev = device is not None and torch.device(device).type != "cpu"
    src = torch.from_numpy(a)
    t = torch.empty(a.shape, dtype=src.dtype, pin_memory=on_dev)
    if t.numel():
        t.copy_(src)
    return t.to(device, non_blocking=True) if on_dev else t


def save_encoded(path: str, encoded, n_fp8_per_stream: int, tile: int = 0,
                 metadata: dict[str, str] | None = None):
    """Store one `tans_codec.encode(...)` result (its 7-tuple)."""
    comp, states, offsets, partial, sm, pair_freqs, spread = encoded
    meta = {"format": FORMAT, "n_fp8_per_stream": int(n_fp8_per_stream), "tile": int(tile),
            "n_streams": int(states.numel()), "block_streams": shard.BLOCK, "table_log": 12}
    meta.update(metadata or {})
    save(path, {"offsets": offsets.to(torch.int32), "pair_freqs": torch.as_tensor(pair_freqs),
                "spread": torch.as_tensor(spread), "states": states, "compressed": comp,
                "partial": partial, "sm": sm}, meta)


def load_encoded(path: str, device=None, rank: int = 0, world: int = 1):
    """The encode 7-tuple stored by `save_encoded`, restricted to this rank's
    encoder blocks (offsets rebased; all of it for world == 1), plus the
    metadata.  pair_freqs and spread stay on the host, as encode returns them."""
    f = _File(path)
    try:
        if f.meta.get("format") != FORMAT:
            raise ValueError(f"{path}: not an encoded-tensor container")
        K = int(f.meta["n_streams"])
        off = f.array("offsets")
        b0, b1 = shard.block_range(K, rank, world)
        s0, s1 = b0 * shard.BLOCK, min(b1 * shard.BLOCK, K)
        lo, hi = int(off[b0]), int(off[b1])
        comp = _to(f.array("compressed")[lo:hi], device)
        offs = _to((off[b0:b1 + 1].astype(np.int64) - lo).astype(np.int32), device)
        states = _to(f.array("states")[s0:s1], device)
        partial = _to(f.array("partial")[s0:s1], device)
        sm = _to(f.array("sm")[:, s0:s1], device)  # the stream axis is dim 1 in both layouts
        pf = torch.from_numpy(f.array("pair_freqs").copy())
        sp = torch.from_numpy(f.array("spread").copy())
        meta = dict(f.meta)
        meta["stream_range"] = f"{s0}:{s1}"
        return (comp, states, offs, partial, sm, pf, sp), meta
    finally:
        f.close()


def save_gemv_weight(path: str, w) -> None:
    """Store a `tans_gemv.EncodedWeight`."""
    save(path, {"offsets": w.offsets.to(torch.int32), "table": w.table, "scale": w.scale.float(),
                "pair_freqs": torch.as_tensor(w.pair_freqs), "spread": torch.as_tensor(w.spread),
                "states": w.states, "compressed": w.compressed, "partial": w.partial, "sm": w.sm},
         {"format": GEMV_FORMAT, "rows": w.rows, "cols": w.cols, "col_splits": w.col_splits,
          "block_streams": shard.BLOCK, "table_log": 12})


def load_gemv_weight(path: str, device=None):
    """The `tans_gemv.EncodedWeight` stored by `save_gemv_weight`."""
    from .tans_gemv import EncodedWeight
    t, meta = load(path, device)
    if meta.get("format") != GEMV_FORMAT:
        raise ValueError(f"{path}: not a GEMV weight container")
    return EncodedWeight(t["compressed"], t["offsets"], t["states"], t["partial"], t["sm"],
                         t["table"], t["scale"], int(meta["rows"]), int(meta["cols"]),
                         int(meta["col_splits"]), t["pair_freqs"].cpu(), t["spread"].cpu())


__all__ = ["save", "load", "save_encoded", "load_encoded", "save_gemv_weight",
           "load_gemv_weight", "FORMAT", "GEMV_FORMAT"]
