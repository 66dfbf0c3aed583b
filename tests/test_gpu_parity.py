"""GPU parity: the sm_100a kernels, called through the C ABI (via the
rans_vectoradd._C binding), against the CPU oracle and against the
reference's own kernels (oracle/_ref, built from the reference sources), on
the reference's own test cases plus edge cases.  Integer/byte work: every
comparison is bit-exact.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from rans_vectoradd import (QWEN3_14B_FP8_EXP, fp8_memcpy, fp8_vecadd_fused_tans,
                            fp8_vecadd_raw, gpu_tans_decode, random_fp8_bytes, tans_codec)
from rans_vectoradd import _C
from rans_vectoradd.data import exponent_histogram, normal_fp8_bytes

pytestmark = pytest.mark.gpu
QWEN = torch.tensor(QWEN3_14B_FP8_EXP, dtype=torch.float64)


def untile(out_flat: torch.Tensor, K: int, N: int) -> torch.Tensor:
    return out_flat.view(N // 16, K, 16).permute(1, 0, 2).reshape(K, N)


def all_pairs(dev):
    i = torch.arange(65536, dtype=torch.int64)
    return ((i // 256).to(torch.uint8).to(dev), (i % 256).to(torch.uint8).to(dev))


# ---------------------------------------------------------------- FP8 add

def test_add_exhaustive_vs_oracle(cuda):
    a, b = all_pairs(cuda)
    got = fp8_vecadd_raw(a, b).cpu().numpy().reshape(256, 256)
    want = oracle.fp8_add_table()
    bad = np.argwhere(got != want)
    assert bad.size == 0, f"{len(bad)} mismatches, first (a,b)={bad[:5].tolist()}"


def test_add_exhaustive_vs_reference_kernel(cuda, ref_ext):
    """The reference raw kernel (f32 add + __nv_fp8_e4m3 satfinite) on all
    65,536 byte pairs: pins the oracle's add and our f16x2 path."""
    a, b = all_pairs(cuda)
    ref = ref_ext.fp8_vecadd_raw(a, b).cpu().numpy().reshape(256, 256)
    assert np.array_equal(ref, oracle.fp8_add_table())
    assert np.array_equal(fp8_vecadd_raw(a, b).cpu().numpy().reshape(256, 256), ref)


@pytest.mark.parametrize("n", [16, 4096 + 16, (1 << 22) + 48])
def test_raw_random_vs_oracle(cuda, n):
    g = torch.Generator().manual_seed(n)
    a = torch.randint(0, 256, (n,), dtype=torch.uint8, generator=g)
    b = torch.randint(0, 256, (n,), dtype=torch.uint8, generator=g)
    got = fp8_vecadd_raw(a.to(cuda), b.to(cuda)).cpu().numpy()
    assert np.array_equal(got, oracle.vecadd_raw(a, b))


def test_raw_keeps_shape(cuda):
    a = torch.zeros((4, 8, 2), dtype=torch.uint8, device=cuda)
    assert fp8_vecadd_raw(a, a).shape == a.shape


@pytest.mark.parametrize("n", [16, 48, (1 << 20) + 16])
def test_memcpy(cuda, n):
    a = torch.randint(0, 256, (n,), dtype=torch.uint8, device=cuda)
    assert torch.equal(fp8_memcpy(a), a)


def test_misaligned_view_rejected(cuda):
    a = torch.zeros(64, dtype=torch.uint8, device=cuda)
    with pytest.raises(RuntimeError, match="aligned"):
        fp8_vecadd_raw(a[1:33], a[1:33])


# ----------------------------------------------------------------- decode

def encode_qwen(K, N, seed, tile=0):
    torch.manual_seed(seed)
    fp8 = random_fp8_bytes(K * N, device="cpu").reshape(K, N)
    return fp8, tans_codec.encode(fp8, QWEN, tile=tile)


@pytest.mark.parametrize("K,N", [(128, 128), (1024, 128), (10_000, 128), (100_000, 128)])
def test_decode_round_trip_reference_cases(cuda, K, N):
    """test_gpu_decode_tans.py:17-48,69-74."""
    fp8, (comp, st, off, part, sm, pf, sp) = encode_qwen(K, N, 42)
    out = gpu_tans_decode(comp.to(cuda), off.to(cuda), st.to(cuda), part.to(cuda),
                          sm.to(cuda), sp.to(cuda), pf.to(cuda), N)
    assert out.shape == (N, K)
    assert torch.equal(out.cpu().t(), fp8)
    assert _C.data_status(cuda) == 0


def test_decode_matches_reference_kernel(cuda, ref_ext):
    fp8, (comp, st, off, part, sm, pf, sp) = encode_qwen(10_000, 256, 7)
    args = [t.to(cuda) for t in (comp, off, st, part, sm, sp, pf)]
    ours = gpu_tans_decode(*args, 256)
    ref = ref_ext.gpu_tans_decode(*args, 256)
    assert torch.equal(ours, ref)


def test_decode_host_table_path(cuda):
    """spread/freqs on the CPU: the table is built on the host (reference path)."""
    fp8, (comp, st, off, part, sm, pf, sp) = encode_qwen(300, 64, 3)
    out = gpu_tans_decode(comp.to(cuda), off.to(cuda), st.to(cuda), part.to(cuda),
                          sm.to(cuda), sp, pf, 64)
    assert torch.equal(out.cpu().t(), fp8)


def test_device_table_build_matches_host(cuda):
    t = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__),
                                            "golden", "tables.npz"))
    for src in ("qwen", "cfg0"):
        sp = torch.from_numpy(t[f"{src}_spread"]).to(cuda)
        pf = torch.from_numpy(t[f"{src}_pair_freqs"]).to(cuda)
        got = _C.build_decode_table_device(sp, pf)
        assert np.array_equal(got.cpu().numpy(), t[f"{src}_table"]), src


@pytest.mark.parametrize("K,N", [(1, 2), (33, 16), (129, 8192), (4096, 2), (517, 1000),
                                 (132, 1002), (96, 18), (256, 4100)])
def test_decode_ragged_vs_oracle(cuda, K, N):
    gen = torch.Generator().manual_seed(K + N)
    fp8 = random_fp8_bytes(K * N, device="cpu", generator=gen).reshape(K, N)
    comp, st, off, part, sm, pf, sp = tans_codec.encode(fp8, QWEN)
    out = gpu_tans_decode(comp.to(cuda), off.to(cuda), st.to(cuda), part.to(cuda),
                          sm.to(cuda), sp.to(cuda), pf.to(cuda), N).cpu().numpy()
    tab = tans_codec.build_decode_table(sp.numpy(), pf.numpy())
    want, ok = oracle.decode(comp, off, st, part, sm, tab, N)
    assert ok and np.array_equal(out, want)
    assert np.array_equal(out.T, fp8.numpy())


@pytest.mark.parametrize("shift", [0, 4, 16])
def test_decode_output_alignment(cuda, shift):
    """K a multiple of 128: a 16-byte aligned output takes the team form
    (16-byte row stores), a 4-byte aligned one the per-warp word form; both
    exact, through the C ABI."""
    from rans_vectoradd._lib import LIB, check
    K, N = 256, 96
    gen = torch.Generator().manual_seed(shift)
    fp8 = random_fp8_bytes(K * N, device="cpu", generator=gen).reshape(K, N)
    comp, st, off, part, sm, pf, sp = tans_codec.encode(fp8, QWEN)
    tab = torch.as_tensor(tans_codec.build_decode_table(sp.numpy(), pf.numpy())).to(cuda)
    d = [t.to(cuda) for t in (comp, off, st, part, sm)]
    buf = torch.zeros(N * K + 64, dtype=torch.uint8, device=cuda)
    out = buf[shift:shift + N * K]
    _C.data_status(cuda)
    check(LIB.tans_b200_decode(d[0].data_ptr(), d[0].numel(), d[1].data_ptr(), d[2].data_ptr(),
                               d[3].data_ptr(), d[4].data_ptr(), tab.data_ptr(), out.data_ptr(),
                               K, N, _C._status(cuda).data_ptr(),
                               torch.cuda.current_stream(cuda).cuda_stream))
    assert _C.data_status(cuda) == 0
    assert torch.equal(out.view(N, K).t().cpu(), fp8)
    assert not buf[:shift].any() and not buf[shift + N * K:].any()


def test_decode_flags_bad_metadata_without_fault(cuda):
    fp8, (comp, st, off, part, sm, pf, sp) = encode_qwen(256, 64, 5)
    _C.data_status(cuda)
    bad_off = off.clone()
    bad_off[0] = -4  # block 0 starts before the buffer; block 1 is untouched
    out = gpu_tans_decode(comp.to(cuda), bad_off.to(cuda), st.to(cuda), part.to(cuda),
                          sm.to(cuda), sp.to(cuda), pf.to(cuda), 64)
    assert _C.data_status(cuda) & 1
    # block 0 is zeroed, block 1 still decodes
    assert torch.equal(out.cpu().t()[128:], fp8[128:])
    assert (out.cpu().t()[:128] == 0).all()
    bad_st = st.clone()
    bad_st[5] = 17
    gpu_tans_decode(comp.to(cuda), off.to(cuda), bad_st.to(cuda), part.to(cuda),
                    sm.to(cuda), sp.to(cuda), pf.to(cuda), 64)
    assert _C.data_status(cuda) & 2
    assert _C.data_status(cuda) == 0


# ------------------------------------------------------------------ fused

def fused_inputs(K, N, seed):
    torch.manual_seed(seed)
    a = random_fp8_bytes(K * N, device="cpu").reshape(K, N)
    b = random_fp8_bytes(K * N, device="cpu").reshape(K, N)
    ca, sa, oa, pa, sma, pf, sp = tans_codec.encode(a, QWEN, tile=8)
    cb, sb, ob, pb, smb, _, _ = tans_codec.encode(b, QWEN, tile=8)
    tbl = tans_codec.build_decode_table(sp.numpy(), pf.numpy())
    return a, b, (ca, oa, sa, pa, sma, cb, ob, sb, pb, smb, tbl)


@pytest.mark.parametrize("K,N", [(1024, 128), (10_000, 256), (1024, 1024)])
def test_fused_equals_raw_reference_cases(cuda, K, N):
    """test_vecadd_tans.py:30-57,76-80: fused == raw, byte for byte."""
    a, b, args = fused_inputs(K, N, 0)
    out = fp8_vecadd_fused_tans(*[t.to(cuda) for t in args], N)
    raw = fp8_vecadd_raw(a.flatten().to(cuda), b.flatten().to(cuda)).reshape(K, N)
    assert torch.equal(untile(out, K, N), raw)
    assert np.array_equal(untile(out, K, N).cpu().numpy(),
                          oracle.vecadd_raw(a, b).reshape(K, N))


def test_fused_matches_reference_kernel(cuda, ref_ext):
    a, b, args = fused_inputs(10_000, 256, 11)
    dargs = [t.to(cuda) for t in args]
    assert torch.equal(fp8_vecadd_fused_tans(*dargs, 256),
                       ref_ext.fp8_vecadd_fused_tans(*dargs, 256))


@pytest.mark.parametrize("K,N", [(1, 16), (31, 16), (129, 2048), (700, 160), (64, 32768)])
def test_fused_ragged_vs_oracle(cuda, K, N):
    gen = torch.Generator().manual_seed(K * 7 + N)
    a = random_fp8_bytes(K * N, device="cpu", generator=gen).reshape(K, N)
    b = random_fp8_bytes(K * N, device="cpu", generator=gen).reshape(K, N)
    ea = tans_codec.encode(a, QWEN, tile=8)
    eb = tans_codec.encode(b, QWEN, tile=8)
    tbl = tans_codec.build_decode_table(ea[6].numpy(), ea[5].numpy())
    args = (ea[0], ea[2], ea[1], ea[3], ea[4], eb[0], eb[2], eb[1], eb[3], eb[4], tbl)
    out = fp8_vecadd_fused_tans(*[t.to(cuda) for t in args], N).cpu().numpy()
    want, ok = oracle.vecadd_fused(args[:5], args[5:10], tbl, N)
    assert ok and np.array_equal(out, want)


def test_fused_cfg0_bit_exact(cuda):
    """cfg0: 2^24 N(0,1) e4m3 per input, 4096-pair streams, shared table."""
    n, N = 1 << 24, 8192
    gen = torch.Generator().manual_seed(0)
    x = normal_fp8_bytes(n, generator=gen)
    y = normal_fp8_bytes(n, generator=gen)
    hist = exponent_histogram(x, y).double()
    K = n // N
    ex = tans_codec.encode(x.reshape(K, N), hist, tile=8)
    ey = tans_codec.encode(y.reshape(K, N), hist, tile=8)
    tbl = tans_codec.build_decode_table(ex[6].numpy(), ex[5].numpy())
    args = [ex[0], ex[2], ex[1], ex[3], ex[4], ey[0], ey[2], ey[1], ey[3], ey[4], tbl]
    out = fp8_vecadd_fused_tans(*[t.to(cuda) for t in args], N)
    raw = fp8_vecadd_raw(x.to(cuda), y.to(cuda)).reshape(K, N)
    assert torch.equal(untile(out, K, N), raw)
    assert np.array_equal(raw.cpu().numpy().ravel(), oracle.vecadd_raw(x, y))


def test_fused_on_side_stream_and_graph(cuda):
    a, b, args = fused_inputs(512, 256, 9)
    dargs = [t.to(cuda) for t in args]
    ref = fp8_vecadd_fused_tans(*dargs, 256)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        out = fp8_vecadd_fused_tans(*dargs, 256)
    s.synchronize()
    assert torch.equal(out, ref)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        gout = fp8_vecadd_fused_tans(*dargs, 256)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(gout, ref)


def test_fused_flags_bad_metadata_without_fault(cuda):
    a, b, args = fused_inputs(256, 64, 13)
    dargs = [t.to(cuda) for t in args]
    _C.data_status(cuda)
    dargs[1] = dargs[1].clone()
    dargs[1][2] = 2 ** 30  # offset beyond the compressed buffer
    out = fp8_vecadd_fused_tans(*dargs, 64)
    assert _C.data_status(cuda) & 1
    good = untile(out, 256, 64)[:128]
    raw = fp8_vecadd_raw(a.flatten().to(cuda), b.flatten().to(cuda)).reshape(256, 64)
    assert torch.equal(good, raw[:128])


def skewed_fp8(K, N, seed):
    """Even streams: one repeated byte (few bits per pair); odd streams:
    exponents uniform over all 16 values (rare pairs cost up to 12 bits).
    Lanes of a warp then drift far apart in their slab rows, which forces the
    kernels' global-refill fallback."""
    g = torch.Generator().manual_seed(seed)
    x = random_fp8_bytes(K * N, device="cpu", generator=g,
                         exp_probs=tuple([1.0] * 16)).reshape(K, N)
    x[0::2] = 0x68  # exponent 13, mantissa 0
    return x


@pytest.mark.parametrize("N", [4096, 32768, 65536])
def test_fused_skewed_streams_fallback(cuda, N):
    K = 96
    a = skewed_fp8(K, N, 1)
    b = skewed_fp8(K, N, 2)
    ea = tans_codec.encode(a, QWEN, tile=8)
    eb = tans_codec.encode(b, QWEN, tile=8)
    tbl = tans_codec.build_decode_table(ea[6].numpy(), ea[5].numpy())
    args = (ea[0], ea[2], ea[1], ea[3], ea[4], eb[0], eb[2], eb[1], eb[3], eb[4], tbl)
    out = fp8_vecadd_fused_tans(*[t.to(cuda) for t in args], N)
    raw = fp8_vecadd_raw(a.flatten().to(cuda), b.flatten().to(cuda)).reshape(K, N)
    assert torch.equal(untile(out, K, N), raw)


@pytest.mark.parametrize("N", [4096, 65536])
def test_decode_skewed_streams_fallback(cuda, N):
    K = 96
    x = skewed_fp8(K, N, 3)
    comp, st, off, part, sm, pf, sp = tans_codec.encode(x, QWEN)
    out = gpu_tans_decode(comp.to(cuda), off.to(cuda), st.to(cuda), part.to(cuda),
                          sm.to(cuda), sp.to(cuda), pf.to(cuda), N)
    assert torch.equal(out.cpu().t(), x)
