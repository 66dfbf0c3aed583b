"""Pin the CPU oracle against the reference's golden vectors (tests/golden/,
generated from the reference itself by tests/golden/make_golden.py) and
against independent e4m3 arithmetic.  CPU only."""
from __future__ import annotations

import hashlib
import os

import numpy as np
import pytest
import torch

import oracle

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def sha(a) -> str:
    a = a.numpy() if hasattr(a, "numpy") else np.asarray(a)
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def small():
    return dict(np.load(os.path.join(GOLDEN, "codec_small.npz")))


def test_decode_table_matches_reference(small):
    tab = oracle.build_decode_table(small["spread"], small["pair_freqs"])
    assert np.array_equal(tab, small["table"])


def test_tables_npz_decode_tables():
    t = np.load(os.path.join(GOLDEN, "tables.npz"))
    for src in ("qwen", "cfg0"):
        tab = oracle.build_decode_table(t[f"{src}_spread"], t[f"{src}_pair_freqs"])
        assert np.array_equal(tab, t[f"{src}_table"]), src


def test_encode_matches_reference_bytes(small):
    fp8 = small["fp8"]
    K, N = fp8.shape
    e = (fp8 >> 3) & 15
    syms = (e[:, 0::2] * 16 + e[:, 1::2]).astype(np.uint8)
    comp, st, off, part = oracle.encode(syms, small["pair_freqs"], small["spread"])
    assert np.array_equal(comp, small["compressed"])
    assert np.array_equal(st, small["states"])
    assert np.array_equal(off, small["offsets"])
    assert np.array_equal(part, small["partial"])


def test_decode_round_trip_of_reference_stream(small):
    fp8 = small["fp8"]
    out, ok = oracle.decode(small["compressed"], small["offsets"], small["states"],
                            small["partial"], small["sm"], small["table"], fp8.shape[1])
    assert ok
    assert np.array_equal(out.T, fp8)


def test_decode_flags_malformed_offsets(small):
    off = small["offsets"].copy()
    off[1] = off[0] + 3  # not a multiple of 512
    _, ok = oracle.decode(small["compressed"], off, small["states"], small["partial"],
                          small["sm"], small["table"], small["fp8"].shape[1])
    assert not ok


def e4m3_values() -> np.ndarray:
    return torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).double().numpy()


def test_e4m3_decode_all_bytes():
    v = e4m3_values()
    for b in range(256):
        got = oracle.lib().oracle_e4m3_to_double(b)
        if np.isnan(v[b]):
            assert np.isnan(got)
        else:
            assert got == v[b] and np.signbit(got) == np.signbit(v[b])


def test_add_table_matches_torch_rounding_in_range():
    """torch's e4m3 cast rounds to nearest even but does not saturate, so it
    is an independent check wherever the exact sum is finite and <= 448."""
    t = oracle.fp8_add_table()
    v = e4m3_values()
    s = v[:, None] + v[None, :]
    ok = ~np.isnan(s) & (np.abs(s) <= 448)
    ref = torch.from_numpy(np.where(ok, s, 0.0)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(t[ok], ref[ok])
    assert ok.sum() > 60000


def test_add_saturates_and_canonicalises_nan():
    t = oracle.fp8_add_table()
    assert t[0x7E, 0x7E] == 0x7E          # 448 + 448 -> 448
    assert t[0xFE, 0xFE] == 0xFE          # -448 + -448 -> -448
    assert t[0x7E, 0x70] == 0x7E          # 448 + 256 saturates
    assert t[0x7F, 0x00] == 0x7F          # NaN in -> 0x7F
    assert t[0xFF, 0x38] == 0x7F          # -NaN + 1 -> 0x7F
    assert t[0x80, 0x80] == 0x80          # -0 + -0 = -0
    assert t[0x80, 0x00] == 0x00          # -0 + +0 = +0
    assert t[0x38, 0xB8] == 0x00          # 1 + -1 = +0
    assert t[0x01, 0x01] == 0x02          # subnormal doubling
    assert t[0x07, 0x01] == 0x08          # subnormal carries into the first normal


def test_add_is_commutative():
    t = oracle.fp8_add_table()
    assert np.array_equal(t, t.T)


def test_fused_equals_raw_on_decoded_inputs(small):
    """oracle fused(A, B) == oracle raw add of the decoded inputs."""
    rng = np.random.default_rng(1)
    fp8 = small["fp8"]
    K, N = fp8.shape
    a = fp8
    b = fp8[rng.permutation(K)]
    enc = []
    for x in (a, b):
        e = (x >> 3) & 15
        syms = (e[:, 0::2] * 16 + e[:, 1::2]).astype(np.uint8)
        sm = (((x >> 4) & 8) | (x & 7)).astype(np.uint8)
        smp = (sm[:, 0::2] | (sm[:, 1::2] << 4)).astype(np.uint8)
        tiled = np.ascontiguousarray(smp.reshape(K, N // 16, 8).transpose(1, 0, 2))
        c, st, off, part = oracle.encode(syms, small["pair_freqs"], small["spread"])
        enc.append((c, off, st, part, tiled))
    out, ok = oracle.vecadd_fused(enc[0], enc[1], small["table"], N)
    assert ok
    untiled = out.reshape(N // 16, K, 16).transpose(1, 0, 2).reshape(K, N)
    assert np.array_equal(untiled, oracle.vecadd_raw(a, b).reshape(K, N))


@pytest.mark.parametrize("tile", [0, 8])
def test_oracle_encode_front_matches_codec(tile):
    """oracle.encode_front (numpy restatement of tans_codec.py:90-143 up to
    the slab encoder) equals the golden-pinned codec front end, including a
    profile with empty exponent bins."""
    import numpy as np
    import torch
    from rans_vectoradd import QWEN3_14B_FP8_EXP, random_fp8_bytes, tans_codec
    g = torch.Generator().manual_seed(11)
    x = random_fp8_bytes(96 * 128, device="cpu", generator=g).view(96, 128)
    for prof in (QWEN3_14B_FP8_EXP, [0.0] * 3 + [1.0] * 13):
        syms, sm, freqs, spread = oracle.encode_front(x.numpy(), prof, tile=tile)
        s2, sm2, _ = tans_codec.split_fp8(x, tile=tile)
        pf = tans_codec.pair_freqs_from_exponents(torch.tensor(prof, dtype=torch.float64))
        assert np.array_equal(syms, s2.numpy()) and np.array_equal(sm, sm2.numpy())
        assert np.array_equal(freqs, pf) and np.array_equal(spread, tans_codec.build_spread(pf))
