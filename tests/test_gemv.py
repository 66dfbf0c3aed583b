"""Fused decode-GEMV: stream layout (CPU) and the sm_100a kernel against the
decode-then-dense fp32 reference, relative error <= 1e-3 (GPU)."""
from __future__ import annotations

import pytest
import torch

from rans_vectoradd import tans_gemv

TOL = 1e-3  # ||y - y_ref||_2 / ||y_ref||_2


def make(R, C, seed):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(R, C, generator=g) * 0.02
    return tans_gemv.quantize_rows(w)


def test_stream_matrix_layout():
    """Element (row, col) lands in the stream/position the kernel expects."""
    R, C, KS = 32, 256, 2
    w8 = torch.arange(R * C, dtype=torch.int64).reshape(R, C)  # unique ids
    sm = tans_gemv.stream_matrix(w8, KS)
    CS = C // KS
    for r in (0, 7, 8, 15, 16, 31):
        for c in (0, 1, 2, 9, 15, 16, 100, 255):
            w, g, ch = r // 16, r % 8, (r % 16) // 8
            k, cc = c // CS, c % CS
            j, rem = cc // 16, cc % 16
            h, t, e = rem // 8, (rem % 8) // 2, rem % 2
            sid = ((w * KS + k) * 2 + ch) * 32 + 4 * g + t
            pos = 4 * j + 2 * h + e
            assert sm[sid, pos].item() == r * C + c


@pytest.mark.parametrize("R,C,KS", [(17408, 5120, 5), (5120, 17408, 17), (8704, 5120, 5),
                                    (2560, 17408, 17), (4352, 5120, 10), (1280, 17408, 34),
                                    (2176, 5120, 20), (640, 17408, 68)])
def test_default_col_splits_for_stack_shards(R, C, KS):
    """Column slices chosen for the cfg3 matrices and their 2-, 4- and 8-way
    row shards: slices of >= 1024 columns while that gives enough warps,
    else 512 and then 256 (the short-slice build covers <= 512); every
    choice divides the columns into whole 64-column chunks."""
    ks = tans_gemv.default_col_splits(R, C)
    assert ks == KS
    assert C % (64 * ks) == 0


def test_quantize_rows_maps_row_max_to_448():
    w8, s = make(16, 64, 0)
    v = w8.view(torch.float8_e4m3fn).float()
    assert torch.allclose(v.abs().amax(dim=1), torch.full((16,), 448.0))


@pytest.mark.gpu
@pytest.mark.parametrize("R,C,B,KS", [(16, 64, 1, 1), (64, 512, 8, 1), (128, 1024, 3, 2),
                                      (256, 4352, 8, 4), (1024, 5120, 8, 1)])
def test_gemv_matches_fp32_reference(cuda, R, C, B, KS):
    w8, s = make(R, C, R + C)
    g = torch.Generator().manual_seed(7)
    x = torch.randn(B, C, generator=g).to(torch.bfloat16)
    enc = tans_gemv.encode_weight(w8, s, col_splits=KS).to(cuda)
    y = tans_gemv.gemv(enc, x.to(cuda))
    ref = tans_gemv.reference_gemv(w8, s, x)
    err = tans_gemv.rel_err(y.cpu(), ref)
    assert err <= TOL, err


@pytest.mark.gpu
def test_gemv_cfg3_full_size(cuda):
    """cfg3: W [17408 x 5120] ~ N(0, 0.02), x bf16 N(0,1), batch 1 and 8."""
    R, C = 17408, 5120
    g = torch.Generator().manual_seed(0)
    w = torch.randn(R, C, generator=g) * 0.02
    w8, s = tans_gemv.quantize_rows(w)
    enc = tans_gemv.encode_weight(w8, s).to(cuda)
    for B in (1, 8):
        x = torch.randn(B, C, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
        y = tans_gemv.gemv(enc, x.to(cuda))
        ref = tans_gemv.reference_gemv(w8.to(cuda), s.to(cuda), x.to(cuda))
        assert tans_gemv.rel_err(y, ref) <= TOL


@pytest.mark.gpu
def test_gemv_down_projection_split(cuda):
    """[5120 x 17408] with 4 column slices (reduced deterministically)."""
    R, C = 5120, 17408
    g = torch.Generator().manual_seed(1)
    w8, s = tans_gemv.quantize_rows(torch.randn(R, C, generator=g) * 0.02)
    enc = tans_gemv.encode_weight(w8, s, col_splits=4).to(cuda)
    x = torch.randn(8, C, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16).to(cuda)
    y1 = tans_gemv.gemv(enc, x)
    y2 = tans_gemv.gemv(enc, x)
    assert torch.equal(y1, y2)
    ref = tans_gemv.reference_gemv(w8.to(cuda), s.to(cuda), x)
    assert tans_gemv.rel_err(y1, ref) <= TOL


@pytest.mark.gpu
def test_gemv_chain_reads_each_input_after_its_producer(cuda):
    """Six GEMVs back to back on one stream, each reading the previous one's
    output (an up/down pair of 8-way row-shard shapes, then the full down
    projection, with and without column slices), no host sync in between.
    Each GEMV starts its weight-side set-up while its predecessor still runs;
    its x must still be read only once that predecessor is done.  Output
    buffers start as NaN, so an early read of x would show up in the result.
    Each step is checked against the fp32 reference on the GPU's own input."""
    shapes = [(2176, 5120, None), (5120, 2176, None), (640, 5120, 1), (5120, 640, 2),
              (17408, 5120, None), (5120, 17408, None)]
    B = 8
    encs = []
    for i, (R, C, KS) in enumerate(shapes):
        w8, s = make(R, C, 100 + i)
        encs.append((tans_gemv.encode_weight(w8, s, col_splits=KS).to(cuda), w8.to(cuda), s.to(cuda)))
    x = torch.randn(B, shapes[0][1], generator=torch.Generator().manual_seed(9))
    x = x.to(torch.bfloat16).to(cuda)
    outs = [torch.full((B, R), float("nan"), dtype=torch.bfloat16, device=cuda)
            for R, _, _ in shapes]
    torch.cuda.synchronize()
    h = x
    for (enc, _, _), out in zip(encs, outs):
        h = tans_gemv.gemv(enc, h, out=out)
    torch.cuda.synchronize()
    h = x
    for (enc, w8, s), y in zip(encs, outs):
        ref = tans_gemv.reference_gemv(w8, s, h)
        assert not torch.isnan(y).any()
        assert tans_gemv.rel_err(y, ref) <= TOL
        h = y


@pytest.mark.gpu
@pytest.mark.parametrize("R,C,B,KS", [(16, 64, 1, 1), (48, 128, 3, 2), (256, 1024, 8, 4),
                                      (17408, 5120, 1, None), (5120, 17408, 8, None)])
def test_gemv_raw_matches_fp32_reference(cuda, R, C, B, KS):
    """The uncompressed e4m3 GEMV (the decode-GEMV's denominator): same
    bound against the fp32 reference; deterministic across calls."""
    w8, s = make(R, C, R + 3 * C)
    x = torch.randn(B, C, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    w8d, sd, xd = w8.to(cuda), s.to(cuda), x.to(cuda)
    y1 = tans_gemv.gemv_raw(w8d, sd, xd, col_splits=KS)
    y2 = tans_gemv.gemv_raw(w8d, sd, xd, col_splits=KS)
    assert torch.equal(y1, y2)
    assert tans_gemv.rel_err(y1, tans_gemv.reference_gemv(w8d, sd, xd)) <= TOL


def test_gemv_raw_rejects_bad_shapes():
    from rans_vectoradd._lib import LIB
    assert LIB.tans_b200_gemv_raw(None, None, None, None, None, 24, 64, 1, 1, None) == 1
    assert b"multiple of 16" in LIB.tans_b200_last_error()
    assert LIB.tans_b200_gemv_raw(None, None, None, None, None, 16, 96, 1, 1, None) == 1
    assert LIB.tans_b200_gemv_raw(None, None, None, None, None, 16, 64, 9, 1, None) == 1
    assert LIB.tans_b200_gemv_raw(None, None, None, None, None, 16, 64, 1, 1, None) == 1
    assert b"null pointer" in LIB.tans_b200_last_error()


def test_gemv_rejects_bad_shapes():
    from rans_vectoradd._lib import LIB
    assert LIB.tans_b200_gemv(None, 0, None, None, None, None, None, None, None, None, None,
                              24, 64, 1, 1, None, None) == 1
    assert b"multiple of 16" in LIB.tans_b200_last_error()
    assert LIB.tans_b200_gemv(None, 0, None, None, None, None, None, None, None, None, None,
                              16, 96, 1, 1, None, None) == 1
    assert LIB.tans_b200_gemv(None, 0, None, None, None, None, None, None, None, None, None,
                              16, 64, 9, 1, None, None) == 1


@pytest.mark.gpu
def test_gemv_device_encoded_weight_matches_host(cuda):
    """encode_weight on a CUDA W (device encoder) gives the host encoder's bytes."""
    w8, s = make(1024, 4352, 9)
    host = tans_gemv.encode_weight(w8, s, col_splits=4)
    dev = tans_gemv.encode_weight(w8.to(cuda), s.to(cuda), col_splits=4)
    for name in ("compressed", "offsets", "states", "partial", "sm", "table", "scale"):
        a, b = getattr(host, name), getattr(dev, name)
        assert b.is_cuda and torch.equal(a, b.cpu()), name
    x = torch.randn(8, 4352, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    assert torch.equal(tans_gemv.gemv(dev, x.to(cuda)), tans_gemv.gemv(host.to(cuda), x.to(cuda)))


@pytest.mark.gpu
@pytest.mark.parametrize("R,C,KS", [(64, 512, 1), (256, 4352, 4), (17408, 5120, 2)])
def test_dense_weight_is_exact(cuda, R, C, KS):
    """The dense decode returns the e4m3 values themselves (as bf16)."""
    w8, s = make(R, C, R * 3 + C)
    enc = tans_gemv.encode_weight(w8.to(cuda), s.to(cuda), col_splits=KS)
    dense = tans_gemv.dense_weight(enc)
    assert torch.equal(dense, w8.to(cuda).view(torch.float8_e4m3fn).to(torch.bfloat16))


@pytest.mark.gpu
@pytest.mark.parametrize("R,C,B", [(1024, 5120, 9), (1024, 5120, 64), (1024, 5120, 512),
                                   (1024, 5120, 2048), (17408, 5120, 512), (1040, 2048, 20)])
def test_gemm_large_batch_matches_reference(cuda, monkeypatch, R, C, B):
    """tans_gemv.gemm at prefill batches runs this library's kernels only
    (every library matmul entry is patched to raise) and matches the fp32
    reference within the GEMV bound; rows % 128 != 0 takes 8-token GEMVs."""
    w8, s = make(R, C, 11 + R)
    enc = tans_gemv.encode_weight(w8.to(cuda), s.to(cuda))
    x = torch.randn(B, C, generator=torch.Generator().manual_seed(B)).to(torch.bfloat16).to(cuda)
    ref = tans_gemv.reference_gemv(w8.to(cuda), s.to(cuda), x)

    def no_library_gemm(*a, **k):
        raise AssertionError("tans_gemv.gemm called a library GEMM")
    for name in ("mm", "matmul", "bmm", "addmm", "einsum"):
        monkeypatch.setattr(torch, name, no_library_gemm)
    monkeypatch.setattr(torch.nn.functional, "linear", no_library_gemm)
    y = tans_gemv.gemm(enc, x)
    torch.cuda.synchronize(cuda)
    monkeypatch.undo()
    assert y.shape == (B, R) and tans_gemv.rel_err(y, ref) <= TOL


@pytest.mark.gpu
@pytest.mark.parametrize("R,C,B,KS", [(128, 512, 16, 1), (256, 1024, 40, 1), (1024, 5120, 64, 5),
                                      (512, 4352, 300, 4), (17408, 5120, 256, None),
                                      (128, 512, 1, 1), (384, 2048, 5, 2), (384, 2048, 600, 2),
                                      (256, 1024, 1000, 1), (17408, 5120, 2048, None)])
def test_gemm_tc_matches_reference(cuda, R, C, B, KS):
    """Decode into shared memory + tcgen05 MMA: rel err within the GEMV bound,
    tokens beyond one 256-token tile and ragged token counts included; above
    256 tokens cluster pairs share each decoded tile (even row-block counts)
    or 256-token tiles decode W again (384 rows: three row blocks)."""
    from rans_vectoradd import _C
    w8, s = make(R, C, R + 7 * C)
    enc = tans_gemv.encode_weight(w8.to(cuda), s.to(cuda), col_splits=KS)
    x = torch.randn(B, C, generator=torch.Generator().manual_seed(B)).to(torch.bfloat16).to(cuda)
    _C.data_status(cuda)
    y = tans_gemv.gemm_tc(enc, x)
    assert _C.data_status(cuda) == 0
    ref = tans_gemv.reference_gemv(w8.to(cuda), s.to(cuda), x)
    assert tans_gemv.rel_err(y, ref) <= TOL


def skewed_weight(R, C, seed):
    """e4m3 rows that alternate between one repeated byte (few bits per pair)
    and exponents uniform over all 16 values (up to 12 bits per pair), NaN
    bytes excluded: the lanes of a warp drift apart in their slab rows and
    the kernels take their register-window refill fallback."""
    from rans_vectoradd.data import random_fp8_bytes
    g = torch.Generator().manual_seed(seed)
    w8 = random_fp8_bytes(R * C, device="cpu", generator=g, exp_probs=tuple([1.0] * 16)).reshape(R, C)
    w8[(w8 & 0x7F) == 0x7F] = 0x7E
    w8[0::2] = 0x38  # 1.0
    return w8, torch.full((R,), 1.0 / 448.0)


@pytest.mark.gpu
@pytest.mark.parametrize("R,C,KS,B", [(256, 8192, 1, 8), (1024, 16384, 2, 3)])
def test_gemv_skewed_rows_fallback(cuda, R, C, KS, B):
    w8, s = skewed_weight(R, C, R + C)
    enc = tans_gemv.encode_weight(w8.to(cuda), s.to(cuda), col_splits=KS)
    x = torch.randn(B, C, generator=torch.Generator().manual_seed(B)).to(torch.bfloat16).to(cuda)
    ref = tans_gemv.reference_gemv(w8.to(cuda), s.to(cuda), x)
    assert tans_gemv.rel_err(tans_gemv.gemv(enc, x), ref) <= TOL
    assert tans_gemv.rel_err(tans_gemv.gemm_tc(enc, x), ref) <= TOL


class _LocalGather:
    """A gather descriptor over local buffers only (one GPU): `world` ranks
    whose gathered buffers and flag arrays all live on this device."""

    def __init__(self, dev, batch, rows, world):
        from rans_vectoradd.peer import GatherDesc
        self._desc = GatherDesc
        self.world = world
        self.bufs = [torch.zeros((batch, rows * world), dtype=torch.bfloat16, device=dev)
                     for _ in range(world)]
        self.flag_arrays = [torch.zeros(world, dtype=torch.int32, device=dev) for _ in range(world)]
        self.y_peers = torch.tensor([b.data_ptr() for b in self.bufs], dtype=torch.int64, device=dev)
        self.flag_peers = torch.tensor([f.data_ptr() for f in self.flag_arrays], dtype=torch.int64,
                                       device=dev)
        self.seq = torch.zeros(1, dtype=torch.int32, device=dev)
        self.done = torch.zeros(1, dtype=torch.int32, device=dev)
        self.views = [self.bufs[0]]

    def descriptor(self, k, col0):
        return self._desc(0, self.world, self.y_peers.data_ptr(), self.bufs[0].shape[1], col0,
                          self.flag_peers.data_ptr(), self.flag_arrays[0].data_ptr(),
                          self.seq.data_ptr(), self.done.data_ptr())


@pytest.mark.gpu
def test_gemv_gather_one_rank_equals_gemv(cuda):
    """World 1: the gathering GEMV publishes to itself; same bits as gemv,
    flag and counter advance by one per call."""
    from rans_vectoradd import _C
    w8, s = make(256, 2048, 5)
    enc = tans_gemv.encode_weight(w8.to(cuda), s.to(cuda), col_splits=2)
    x = torch.randn(3, 2048, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16).to(cuda)
    g = _LocalGather(cuda, 3, 256, 1)
    _C.data_status(cuda)
    for step in (1, 2):
        y = tans_gemv.gemv_gather(enc, x, g, 0, 0)
        assert torch.equal(y.view(torch.int16), tans_gemv.gemv(enc, x).view(torch.int16))
        assert int(g.seq.item()) == step and int(g.flag_arrays[0][0].item()) == step
    assert _C.data_status(cuda) == 0


@pytest.mark.gpu
def test_gemv_gather_wait_runs_out_without_hang(cuda):
    """A peer that never publishes: the GEMV's bounded wait gives up (about a
    second per flag), the kernel returns and reports TANS_B200_DATA_TIMEOUT."""
    import time
    from rans_vectoradd import _C
    w8, s = make(128, 512, 6)
    enc = tans_gemv.encode_weight(w8.to(cuda), s.to(cuda), col_splits=1)
    x = torch.randn(1, 512, generator=torch.Generator().manual_seed(6)).to(torch.bfloat16).to(cuda)
    g = _LocalGather(cuda, 1, 128, 2)
    g.seq.fill_(1)  # this rank has "published" once; no peer ever has
    _C.data_status(cuda)
    t0 = time.time()
    tans_gemv.gemv_gather(enc, x, g, 0, 0)
    st = _C.data_status(cuda)
    assert st & 8, f"status {st}: the wait did not report running out"
    assert time.time() - t0 < 30
