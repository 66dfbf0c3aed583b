"""GPU parity of the device slab encoder (csrc/encode.cu) through the C ABI:
byte-identical to the reference's outputs (golden digests of its own test
cases), to the CPU encoder and to the oracle, on the reference's cases plus
ragged, misaligned, empty and error cases; and a full-size encode -> decode
round trip.  Integer/byte work: every comparison is exact.
"""
from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

import oracle
from rans_vectoradd import QWEN3_14B_FP8_EXP, _C, gpu_tans_decode, random_fp8_bytes, tans_codec
from rans_vectoradd._lib import ENC_INPUT_FP8
from rans_vectoradd.data import exponent_histogram, normal_fp8_bytes

pytestmark = pytest.mark.gpu
QWEN = torch.tensor(QWEN3_14B_FP8_EXP, dtype=torch.float64)
NAMES = ["compressed", "states", "offsets", "partial", "sm", "pair_freqs", "spread"]


def sha(t) -> str:
    a = t.cpu().numpy() if hasattr(t, "cpu") else np.asarray(t)
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def qwen_tables():
    pf = tans_codec.pair_freqs_from_exponents(QWEN)
    return torch.from_numpy(pf), torch.from_numpy(tans_codec.build_spread(pf))


def assert_same(dev_out, cpu_out):
    for name, d, c in zip(NAMES, dev_out, cpu_out):
        assert d.dtype == c.dtype, name
        assert torch.equal(d.cpu(), c.cpu()), name


@pytest.mark.parametrize("K,N", [(128, 128), (1024, 128), (10_000, 128), (100_000, 128)])
def test_device_encode_reference_decode_cases(cuda, golden_digests, K, N):
    """test_gpu_decode_tans.py:17-25 inputs (seed 42, Qwen profile, tile 0)."""
    g = golden_digests[f"decode_K{K}_N{N}"]
    torch.manual_seed(42)
    fp8 = random_fp8_bytes(K * N, device="cpu").reshape(K, N)
    out = tans_codec.encode(fp8.to(cuda), QWEN)
    assert all(t.is_cuda for t in out[:5])
    for name, t in zip(NAMES, out):
        assert sha(t) == g[name], name


@pytest.mark.parametrize("K,N", [(1024, 128), (10_000, 256), (1024, 1024)])
def test_device_encode_reference_fused_cases(cuda, golden_digests, K, N):
    """test_vecadd_tans.py:30-38 inputs (seed 0, two inputs, tile 8)."""
    g = golden_digests[f"fused_K{K}_N{N}"]
    torch.manual_seed(0)
    a = random_fp8_bytes(K * N, device="cpu").reshape(K, N)
    b = random_fp8_bytes(K * N, device="cpu").reshape(K, N)
    for x, gg in ((a, g["a"]), (b, g["b"])):
        for name, t in zip(NAMES, tans_codec.encode(x.to(cuda), QWEN, tile=8)):
            assert sha(t) == gg[name], name


def test_device_encode_cfg0(cuda, golden_digests):
    g = golden_digests["cfg0"]
    gen = torch.Generator().manual_seed(0)
    x = normal_fp8_bytes(g["n"], generator=gen)
    y = normal_fp8_bytes(g["n"], generator=gen)
    hist = exponent_histogram(x, y).double()
    for v, gg in ((x, g["x"]), (y, g["y"])):
        out = tans_codec.encode(v.reshape(g["K"], g["N"]).to(cuda), hist, tile=8)
        for name, t in zip(NAMES, out):
            assert sha(t) == gg[name], name


@pytest.mark.parametrize("K,N,tile", [(1, 2, 0), (33, 30, 0), (129, 48, 8), (130, 200, 4),
                                      (300, 1000, 0), (257, 4112, 8), (5, 16 * 9, 0),
                                      (64, 256, 4)])
def test_device_encode_ragged_vs_cpu(cuda, K, N, tile):
    gen = torch.Generator().manual_seed(K * 7 + N)
    fp8 = random_fp8_bytes(K * N, device="cpu", generator=gen).reshape(K, N)
    assert_same(tans_codec.encode(fp8.to(cuda), QWEN, tile=tile),
                tans_codec.encode(fp8, QWEN, tile=tile))


def test_device_encode_misaligned_input(cuda):
    """A 1-byte-offset view takes the unchunked path; bytes are the same."""
    K, N = 200, 256
    gen = torch.Generator().manual_seed(11)
    fp8 = random_fp8_bytes(K * N, device="cpu", generator=gen).reshape(K, N)
    store = torch.empty(K * N + 16, dtype=torch.uint8, device=cuda)
    view = store[1:1 + K * N].view(K, N)
    view.copy_(fp8.to(cuda))
    assert view.data_ptr() % 16 == 1
    for tile in (0, 8):
        assert_same(tans_codec.encode(view, QWEN, tile=tile), tans_codec.encode(fp8, QWEN, tile=tile))


@pytest.mark.parametrize("K,P", [(1, 1), (127, 30), (129, 2), (300, 1000), (64, 4096), (3, 13)])
def test_device_encode_symbols_vs_oracle(cuda, K, P):
    """tans_encode_interleaved on CUDA symbols: same bytes as the oracle."""
    gen = torch.Generator().manual_seed(K * 1000 + P)
    fp8 = random_fp8_bytes(K * 2 * P, device="cpu", generator=gen).reshape(K, 2 * P)
    e = (fp8 >> 3) & 15
    syms = (e[:, 0::2] * 16 + e[:, 1::2]).contiguous()
    pf, sp = qwen_tables()
    got = _C.tans_encode_interleaved(syms.to(cuda), pf, sp)
    want = oracle.encode(syms, pf.numpy(), sp.numpy())
    for g_, w_ in zip(got, want):
        assert g_.is_cuda
        assert np.array_equal(g_.cpu().numpy(), w_)


def test_device_encode_empty_and_zero_length(cuda):
    pf, sp = qwen_tables()
    comp, st, off, part = _C.tans_encode_interleaved(
        torch.empty((0, 16), dtype=torch.uint8, device=cuda), pf, sp)
    assert comp.numel() == 0 and st.numel() == 0 and off.cpu().tolist() == [0]
    syms = torch.empty((130, 0), dtype=torch.uint8)
    got = _C.tans_encode_interleaved(syms.to(cuda), pf, sp)
    want = _C.tans_encode_interleaved(syms, pf, sp)
    for g_, w_ in zip(got, want):
        assert torch.equal(g_.cpu(), w_)


def test_device_encode_single_symbol(cuda):
    f = np.zeros(256, np.int32)
    f[0x77] = 4096
    sp = tans_codec.build_spread(f)
    syms = torch.full((130, 64), 0x77, dtype=torch.uint8)
    got = _C.tans_encode_interleaved(syms.to(cuda), torch.from_numpy(f), torch.from_numpy(sp))
    want = _C.tans_encode_interleaved(syms, torch.from_numpy(f), torch.from_numpy(sp))
    for g_, w_ in zip(got, want):
        assert torch.equal(g_.cpu(), w_)


def test_device_encode_rejects_uncodable_symbol(cuda):
    """Same error as the CPU encoder (the reference loops forever here)."""
    f = np.zeros(256, np.int32)
    f[1] = 4096
    sp = torch.from_numpy(tans_codec.build_spread(f))
    syms = torch.zeros((300, 40), dtype=torch.uint8)
    syms[200, 7] = 1
    syms[5, 3] = 9
    with pytest.raises(RuntimeError, match="symbol 0 occurs but has zero frequency"):
        _C.tans_encode_interleaved(syms.to(cuda), torch.from_numpy(f), sp)
    pf, spq = qwen_tables()
    bad = pf.clone()
    bad[0] += 1
    with pytest.raises(RuntimeError, match="freqs must sum to L=4096"):
        _C.tans_encode_interleaved(syms.to(cuda), bad, spq)
    with pytest.raises(RuntimeError, match="spread"):
        _C.tans_encode_interleaved(syms.to(cuda), pf, torch.zeros(4096, dtype=torch.int32))


def test_device_encode_odd_fp8_rejected(cuda):
    pf, sp = qwen_tables()
    with pytest.raises(RuntimeError, match="even"):
        _C.encode_device(torch.zeros((4, 7), dtype=torch.uint8, device=cuda), ENC_INPUT_FP8,
                         pf, sp)


def test_device_encode_matches_cpu_2e26(cuda):
    """2^26 N(0,1) e4m3 bytes, 4096-pair streams, tile 8 (the vecadd workload's
    format): device and CPU encoders agree byte for byte."""
    gen = torch.Generator().manual_seed(3)
    x = normal_fp8_bytes(1 << 26, generator=gen).reshape(-1, 8192)
    hist = exponent_histogram(x, x).double()
    assert_same(tans_codec.encode(x.to(cuda), hist, tile=8), tans_codec.encode(x, hist, tile=8))


def test_device_encode_decode_round_trip_2e30(cuda):
    """Full-size property: 2^30 e4m3 bytes encoded on the device, decoded on
    the device, equal the input (tile 0, 8192 bytes per stream)."""
    gen = torch.Generator(device=cuda).manual_seed(5)
    x = torch.randn(1 << 30, generator=gen, device=cuda, dtype=torch.float32)
    x = (x * (448.0 / x.abs().max())).to(torch.float8_e4m3fn).view(torch.uint8)
    x = x.reshape(-1, 8192)
    hist = torch.bincount(((x.reshape(-1) >> 3) & 15).long(), minlength=16).cpu().double()
    comp, st, off, part, sm, pf, sp = tans_codec.encode(x, hist)
    out = gpu_tans_decode(comp, off, st, part, sm, sp.to(cuda), pf.to(cuda), 8192)
    assert torch.equal(out.t(), x)
