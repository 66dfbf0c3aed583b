"""Property-based tests (hypothesis) of the host codec against the oracle:
random stream counts and lengths (ragged blocks included), tiles, split
segments and exponent profiles; every encode must equal the oracle's
restatement of the reference encoder byte for byte and decode back to its
input.  CPU only; example counts are kept small so the suite stays fast."""
from __future__ import annotations

import numpy as np
import torch
from hypothesis import given, settings, strategies as st

import oracle
from rans_vectoradd import tans_codec


def _profile(draw_w):
    w = np.asarray(draw_w, dtype=np.float64)
    return torch.tensor(w / w.sum())


@settings(max_examples=25, deadline=None)
@given(K=st.integers(1, 300), P=st.integers(1, 40), seed=st.integers(0, 2**31 - 1),
       weights=st.lists(st.floats(0.05, 10.0), min_size=16, max_size=16))
def test_encode_matches_oracle_and_round_trips(K, P, seed, weights):
    rng = np.random.default_rng(seed)
    prof = _profile(weights)
    exps = rng.choice(16, size=(K, 2 * P), p=prof.numpy())
    sm = rng.integers(0, 16, size=(K, 2 * P))
    fp8 = torch.from_numpy(((sm & 8) << 4 | exps << 3 | (sm & 7)).astype(np.uint8))
    comp, st_, off, part, smp, pf, sp = tans_codec.encode(fp8, prof)
    e = (fp8 >> 3) & 15
    syms = (e[:, 0::2] * 16 + e[:, 1::2]).contiguous()
    want = oracle.encode(syms, pf.numpy(), sp.numpy())
    for got, w in zip((comp, st_, off, part), want):
        assert np.array_equal(got.numpy(), w)
    tab = tans_codec.build_decode_table(sp.numpy(), pf.numpy())
    out, ok = oracle.decode(comp, off, st_, part, smp, tab, 2 * P)
    assert ok and np.array_equal(out.T, fp8.numpy())


@settings(max_examples=15, deadline=None)
@given(K=st.integers(1, 200), segs=st.integers(1, 4), S8=st.integers(1, 4),
       seed=st.integers(0, 2**31 - 1))
def test_split_streams_equal_rearranged_plain_encode(K, segs, S8, seed):
    S = 8 * S8
    P = S * segs
    rng = np.random.default_rng(seed)
    fp8 = torch.from_numpy(rng.integers(0, 256, size=(K, 2 * P), dtype=np.uint8))
    prof = torch.ones(16, dtype=torch.float64)  # every pair symbol gets 16 slots
    split = tans_codec.encode(fp8, prof, tile=8, segment_pairs=S)
    rearranged = fp8.view(K, segs, 2 * S).transpose(0, 1).reshape(segs * K, 2 * S).contiguous()
    plain = tans_codec.encode(rearranged, prof, tile=8)
    for a, b in zip(split[:4], plain[:4]):
        assert torch.equal(a, b)
    assert torch.equal(split[4], tans_codec.encode(fp8, prof, tile=8)[4])
