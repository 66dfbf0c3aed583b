"""Fused tANS-decode GEMV: y = bf16(scale * (e4m3 W) @ x^T), fp32 accumulate.

No counterpart in the reference (it is the GEMV configuration of the
benchmark); it reuses the reference's codec unchanged — same pair symbols,
table, slab layout and encoder — and only chooses which weight elements form
each stream:

* W [rows, cols] e4m3 bytes with a per-row fp32 scale (row max -> 448);
* rows are taken 16 at a time and columns in `col_splits` slices; each
  16-row group x slice is 64 streams: stream ((w*KS + k)*2 + chain)*32 + lane
  holds row 16w + lane//4 + 8*chain and, of every 16-column chunk of the
  slice, columns 2t, 2t+1, 8+2t, 9+2t (t = lane % 4) — the operand layout of
  a 16x8x16 tensor-core fragment, so the kernel turns each decoded pair
  straight into a fragment register.

`encode_weight` builds that stream matrix and encodes it with
`tans_codec.encode(..., tile=8)` (on the GPU when W is a CUDA tensor);
`gemv` runs the sm_100a kernel.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import tans_codec
from ._C import _req, _same_device, _status, _stream
from ._lib import LIB, check


@dataclass
class EncodedWeight:
    compressed: torch.Tensor
    offsets: torch.Tensor
    states: torch.Tensor
    partial: torch.Tensor
    sm: torch.Tensor
    table: torch.Tensor
    scale: torch.Tensor
    rows: int
    cols: int
    col_splits: int
    pair_freqs: torch.Tensor
    spread: torch.Tensor

    def to(self, device) -> "EncodedWeight":
        mv = lambda t: t.to(device)  # noqa: E731
        return EncodedWeight(mv(self.compressed), mv(self.offsets), mv(self.states),
                             mv(self.partial), mv(self.sm), mv(self.table), mv(self.scale),
                             self.rows, self.cols, self.col_splits, self.pair_freqs,
                             self.spread)

    def stream_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in
                   (self.compressed, self.offsets, self.states, self.partial, self.sm))


def quantize_rows(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 W -> (e4m3 bytes, per-row fp32 scale) with row max|w| -> 448."""
    w = w.float()
    scale = w.abs().amax(dim=1).clamp_min(torch.finfo(torch.float32).tiny) / 448.0
    w8 = (w / scale[:, None]).to(torch.float8_e4m3fn).view(torch.uint8)
    return w8, scale


def stream_matrix(w8: torch.Tensor, col_splits: int = 1) -> torch.Tensor:
    """Reorder e4m3 bytes [rows, cols] into the GEMV stream matrix
    [rows*4*col_splits, cols/col_splits/4] (see module docstring)."""
    R, C = w8.shape
    KS = col_splits
    assert R % 16 == 0 and C % (64 * KS) == 0, "rows % 16 and cols % (64*col_splits) must be 0"
    CS = C // KS
    v = w8.reshape(R // 16, 2, 8, KS, CS // 16, 2, 4, 2)   # w c g k j h t e
    return v.permute(0, 3, 1, 2, 6, 4, 5, 7).reshape(R * 4 * KS, CS // 4).contiguous()


def default_col_splits(rows: int, cols: int, sms: int = 148, warps_per_sm: int = 40,
                       min_warps_per_sm: int = 16) -> int:
    """Column slices (one GEMV warp per 16-row group and slice).  First the
    most slices up to about `warps_per_sm` warps per SM with slices of at
    least 1024 columns (shorter streams spend more on per-stream setup);
    if that leaves fewer than `min_warps_per_sm` warps per SM (row shards of
    a multi-GPU stack), the fewest slices of at least 512, then 256, columns
    that reach it.  Slices are multiples of 64 columns.  On B200 at batch 8:
    [17408 x 5120] -> 5, [5120 x 17408] -> 17, [4352 x 5120] -> 10 (25 us vs
    33 us with 5), [1280 x 17408] -> 34 (27 vs 33 us with 17), [640 x 17408]
    -> 68 (21 vs 33 us with 17)."""
    groups = max(1, rows // 16)
    ok = lambda ks, min_cs: cols % (64 * ks) == 0 and cols // ks >= min_cs  # noqa: E731
    want = max(1, round(sms * warps_per_sm / groups))
    ks = max([k for k in range(1, want + 1) if ok(k, 1024)], default=1)
    for min_cs in (512, 256):
        if groups * ks >= sms * min_warps_per_sm:
            break
        more = [k for k in range(ks + 1, cols // 64 + 1) if ok(k, min_cs)]
        hit = [k for k in more if groups * k >= sms * min_warps_per_sm]
        ks = hit[0] if hit else (more[-1] if more else ks)
    return ks


def encode_weight(w8: torch.Tensor, scale: torch.Tensor, exp_freqs=None,
                  col_splits: int | None = None) -> EncodedWeight:
    """tANS-encode e4m3 weight bytes for `gemv`: on the host for a CPU w8,
    with the device encoder (outputs on w8's device) for a CUDA w8; the bytes
    are the same.  `col_splits` defaults to default_col_splits(rows, cols)."""
    w8 = w8.detach().contiguous()
    if col_splits is None:
        col_splits = default_col_splits(*w8.shape)
    if exp_freqs is None:
        # empty exponent bins get weight 1 so every pair keeps a slot (no
        # zero-probability symbols for the frequency quantiser to misplace)
        exp_freqs = torch.bincount(((w8.reshape(-1) >> 3) & 15).long(),
                                   minlength=16).clamp_min(1).double().cpu()
    streams = stream_matrix(w8, col_splits)
    comp, st, off, part, sm, pf, sp = tans_codec.encode(streams, exp_freqs, tile=8)
    table = tans_codec.build_decode_table(sp.numpy(), pf.numpy()).to(w8.device)
    return EncodedWeight(comp, off, st, part, sm, table,
                         scale.detach().float().to(w8.device).contiguous(), w8.shape[0],
                         w8.shape[1], col_splits, pf, sp)


def gemv(weight: EncodedWeight, x: torch.Tensor, out: torch.Tensor | None = None,
         partials: torch.Tensor | None = None) -> torch.Tensor:
    """y [batch, rows] bf16 = scale * W @ x^T for x bf16 [batch, cols], batch 1..8.
    All of `weight` and x must be CUDA tensors on one device."""
    _req(x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 2 and x.is_contiguous(),
         "x must be a contiguous CUDA bfloat16 [batch, cols] tensor")
    B, C = x.shape
    _req(C == weight.cols, f"x has {C} columns, the weight {weight.cols}")
    _req(1 <= B <= 8, "batch must be 1..8")
    dev = x.device
    _same_device(dev, weight.compressed, weight.offsets, weight.states, weight.partial,
                 weight.sm, weight.table, weight.scale)
    R, KS = weight.rows, weight.col_splits
    with torch.cuda.device(dev):
        if out is None:
            out = torch.empty((B, R), dtype=torch.bfloat16, device=dev)
        if KS > 1 and partials is None:
            partials = torch.empty((KS, B, R), dtype=torch.float32, device=dev)
        check(LIB.tans_b200_gemv(
            weight.compressed.data_ptr(), weight.compressed.numel(), weight.offsets.data_ptr(),
            weight.states.data_ptr(), weight.partial.data_ptr(), weight.sm.data_ptr(),
            weight.table.data_ptr(), weight.scale.data_ptr(), x.data_ptr(), out.data_ptr(),
            partials.data_ptr() if partials is not None else None, R, C, B, KS,
            _status(dev).data_ptr(), _stream(dev)))
    return out


def gemv_gather(weight: EncodedWeight, x: torch.Tensor, gather, k: int, col0: int,
                partials: torch.Tensor | None = None) -> torch.Tensor:
    """This rank's row shard of a GEMV (rows col0 .. col0 + weight.rows of the
    full output), stored into every rank's gathered buffer `gather.views[k]`
    by the GEMV epilogue itself (rans_vectoradd.peer.PeerGather); returns
    this rank's view of the gathered [batch, width] output.  The kernel
    first waits for every rank's previous gather, so x may be a gathered
    buffer of an earlier step, but never `gather.views[k]` itself (or any
    tensor sharing its memory): a faster peer's epilogue of this step may
    already be writing there while this rank's GEMV still reads x.
    Consecutive gathers must therefore alternate between buffers."""
    _req(x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 2 and x.is_contiguous(),
         "x must be a contiguous CUDA bfloat16 [batch, cols] tensor")
    B, C = x.shape
    _req(C == weight.cols, f"x has {C} columns, the weight {weight.cols}")
    _req(1 <= B <= 8, "batch must be 1..8")
    out = gather.views[k]
    _req(out.shape[0] == B, f"gathered buffer holds batch {out.shape[0]}, x has {B}")
    xs, xe = x.data_ptr(), x.data_ptr() + x.numel() * x.element_size()
    os_, oe = out.data_ptr(), out.data_ptr() + out.numel() * out.element_size()
    _req(xe <= os_ or oe <= xs,
         f"x overlaps the gathered buffer views[{k}] that this GEMV writes; "
         "use a different gathered buffer for consecutive gathers")
    dev = x.device
    _same_device(dev, weight.compressed, weight.offsets, weight.states, weight.partial,
                 weight.sm, weight.table, weight.scale, out)
    R, KS = weight.rows, weight.col_splits
    with torch.cuda.device(dev):
        if partials is None:
            partials = torch.empty((KS, B, R), dtype=torch.float32, device=dev)
        _req(partials.numel() >= KS * B * R and partials.dtype == torch.float32,
             "partials must be f32 with col_splits * batch * rows elements")
        desc = gather.descriptor(k, col0)
        check(LIB.tans_b200_gemv_gather(
            weight.compressed.data_ptr(), weight.compressed.numel(), weight.offsets.data_ptr(),
            weight.states.data_ptr(), weight.partial.data_ptr(), weight.sm.data_ptr(),
            weight.table.data_ptr(), weight.scale.data_ptr(), x.data_ptr(), partials.data_ptr(),
            R, C, B, KS, ctypes.addressof(desc), _status(dev).data_ptr(), _stream(dev)))
    return out


def dense_weight(weight: EncodedWeight, out: torch.Tensor | None = None) -> torch.Tensor:
    """Decode a CUDA EncodedWeight to a dense row-major bf16 [rows, cols]
    matrix of its e4m3 values (unscaled; e4m3 -> bf16 is exact)."""
    dev = weight.compressed.device
    _req(weight.compressed.is_cuda, "weight must be on a CUDA device")
    _same_device(dev, weight.offsets, weight.states, weight.partial, weight.sm, weight.table)
    R, C = weight.rows, weight.cols
    with torch.cuda.device(dev):
        if out is None:
            out = torch.empty((R, C), dtype=torch.bfloat16, device=dev)
        _req(out.shape == (R, C) and out.dtype == torch.bfloat16 and out.is_contiguous()
             and out.device == dev, "out must be a contiguous bf16 [rows, cols] tensor")
        check(LIB.tans_b200_gemv_weight_dense(
            weight.compressed.data_ptr(), weight.compressed.numel(), weight.offsets.data_ptr(),
            weight.states.data_ptr(), weight.partial.data_ptr(), weight.sm.data_ptr(),
            weight.table.data_ptr(), out.data_ptr(), R, C, weight.col_splits,
            _status(dev).data_ptr(), _stream(dev)))
    return out


# Largest batch sent to `gemm_tc` by `gemm`: it decodes the weight once per
# 256-token tile, so beyond one tile the dense decode + library GEMM is
# faster (on B200, [17408 x 5120]: 116 us vs 139 us at 256 tokens, 229 us vs
# 158 us at 512).
def gemm(weight: EncodedWeight, x: torch.Tensor) -> torch.Tensor:
    """y [batch, rows] bf16 = scale * W @ x^T for any batch, on this
    library's own kernels only: the fused GEMV kernel up to 8 tokens; above
    that the fused decode + tensor-core kernel (`gemm_tc`, every token count)
    when rows % 128 == 0, else the GEMV kernel over 8-token slices of x.  The
    dense form (`gemm_dense`: dense bf16 decode + a library GEMM) is a
    separate entry point and is never chosen here."""
    _req(x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 2 and x.is_contiguous(),
         "x must be a contiguous CUDA bfloat16 [batch, cols] tensor")
    if x.shape[0] <= 8:
        return gemv(weight, x)
    if weight.rows % 128 == 0:
        return gemm_tc(weight, x if x.data_ptr() % 16 == 0 else x.clone())
    return torch.cat([gemv(weight, x[i:i + 8]) for i in range(0, x.shape[0], 8)])


def gemm_dense(weight: EncodedWeight, x: torch.Tensor, w_dense: torch.Tensor | None = None
               ) -> torch.Tensor:
    """The large-batch form of `gemm`: dense bf16 decode of W (or `w_dense`),
    library bf16 GEMM with fp32 output, per-row scale, one rounding."""
    _req(x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 2 and x.is_contiguous(),
         "x must be a contiguous CUDA bfloat16 [batch, cols] tensor")
    w = dense_weight(weight) if w_dense is None else w_dense
    acc = torch.mm(x, w.t(), out_dtype=torch.float32)
    R = weight.rows
    dev = x.device
    with torch.cuda.device(dev):
        y = torch.empty((x.shape[0], R), dtype=torch.bfloat16, device=dev)
        check(LIB.tans_b200_scale_rows_bf16(acc.data_ptr(), weight.scale.data_ptr(), y.data_ptr(),
                                            x.shape[0], R, _stream(dev)))
    return y


def gemm_tc(weight: EncodedWeight, x: torch.Tensor, out: torch.Tensor | None = None
            ) -> torch.Tensor:
    """y [batch, rows] bf16 = scale * W @ x^T on the tensor cores with W
    decoded on the fly into shared memory (tcgen05; rows % 128 == 0)."""
    _req(x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 2 and x.is_contiguous(),
         "x must be a contiguous CUDA bfloat16 [batch, cols] tensor")
    B, C = x.shape
    _req(C == weight.cols, f"x has {C} columns, the weight {weight.cols}")
    dev = x.device
    _same_device(dev, weight.compressed, weight.offsets, weight.states, weight.partial,
                 weight.sm, weight.table, weight.scale)
    with torch.cuda.device(dev):
        if out is None:
            out = torch.empty((B, weight.rows), dtype=torch.bfloat16, device=dev)
        check(LIB.tans_b200_gemm_tc(
            weight.compressed.data_ptr(), weight.compressed.numel(), weight.offsets.data_ptr(),
            weight.states.data_ptr(), weight.partial.data_ptr(), weight.sm.data_ptr(),
            weight.table.data_ptr(), weight.scale.data_ptr(), x.data_ptr(), out.data_ptr(),
            weight.rows, C, weight.col_splits, B, _status(dev).data_ptr(), _stream(dev)))
    return out


def raw_col_splits(rows: int, cols: int, sms: int = 148) -> int:
    """Column slices of the uncompressed GEMV: the fewest that divide the
    64-column chunks and give about 4.5 CTAs (128 rows each) per SM (best of
    a sweep over slices and grid shapes on [17408 x 5120] and [5120 x 17408])."""
    chunks = cols // 64
    for d in range(1, chunks + 1):
        if chunks % d == 0 and (rows + 127) // 128 * d * 2 >= 9 * sms:
            return d
    return chunks


def gemv_raw(w8: torch.Tensor, scale: torch.Tensor, x: torch.Tensor,
             out: torch.Tensor | None = None, partials: torch.Tensor | None = None,
             col_splits: int | None = None) -> torch.Tensor:
    """Uncompressed e4m3 GEMV, y = bf16(scale * (W8 @ x^T)) with fp32
    accumulate (no reference counterpart): the same mma.sync path and column
    reduction as gemv() with the weight read as plain e4m3 bytes, i.e. the
    decode-GEMV's denominator.  w8: uint8 (e4m3 bits) [rows, cols] on CUDA."""
    _req(w8.is_cuda and w8.dtype == torch.uint8 and w8.dim() == 2 and w8.is_contiguous(),
         "w8 must be a contiguous CUDA uint8 [rows, cols] tensor of e4m3 bits")
    _req(x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 2 and x.is_contiguous(),
         "x must be a contiguous CUDA bfloat16 [batch, cols] tensor")
    if x.data_ptr() % 16:
        x = x.clone()  # 16-byte aligned copy for the vector loads
    R, C = w8.shape
    B = x.shape[0]
    _req(x.shape[1] == C, f"x has {x.shape[1]} columns, the weight {C}")
    _req(1 <= B <= 8, "batch must be 1..8")
    dev = w8.device
    _same_device(dev, scale, x)
    KS = col_splits or raw_col_splits(R, C)
    with torch.cuda.device(dev):
        if out is None:
            out = torch.empty((B, R), dtype=torch.bfloat16, device=dev)
        if partials is None:
            partials = torch.empty((KS, B, R), dtype=torch.float32, device=dev)
        _req(partials.numel() >= KS * B * R and partials.dtype == torch.float32,
             "partials must be f32 with col_splits * batch * rows elements")
        sc = scale.float().contiguous()
        check(LIB.tans_b200_gemv_raw(w8.data_ptr(), sc.data_ptr(), x.data_ptr(), out.data_ptr(),
                                     partials.data_ptr(), R, C, B, KS, _stream(dev)))
    return out


def reference_gemv(w8: torch.Tensor, scale: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """Decode-then-dense fp32 reference: bf16((W8.float() * s) @ x.float()^T)."""
    w = w8.view(torch.float8_e4m3fn).float() * scale.float()[:, None]
    return (x.float() @ w.t()).to(torch.bfloat16)


def rel_err(y: torch.Tensor, y_ref: torch.Tensor) -> float:
    a, b = y.float(), y_ref.float()
    return float(torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b).clamp_min(1e-30))


__all__ = ["EncodedWeight", "quantize_rows", "stream_matrix", "encode_weight", "gemv",
           "dense_weight", "gemm", "gemm_tc", "reference_gemv", "rel_err"]
