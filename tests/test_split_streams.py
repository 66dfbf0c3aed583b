"""Split-stream format extension (segment_pairs): every stream of P pair
symbols is encoded as P/S sub-streams, segment-major.  Its bytes are the
reference encoder's bytes for the rearranged pair-symbol matrix (pinned here
against the oracle's restatement of that encoder); decoding and the fused add
on it reproduce the unsplit results bit for bit."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from rans_vectoradd import (QWEN3_14B_FP8_EXP, fp8_vecadd_fused_tans, fp8_vecadd_raw,
                            gpu_tans_decode, random_fp8_bytes, tans_codec)

QWEN = torch.tensor(QWEN3_14B_FP8_EXP, dtype=torch.float64)


def inputs(K, N, seed):
    g = torch.Generator().manual_seed(seed)
    return random_fp8_bytes(K * N, device="cpu", generator=g).reshape(K, N)


def split_syms(x, S):
    K, N = x.shape
    e = (x >> 3) & 15
    syms = (e[:, 0::2] * 16 + e[:, 1::2])
    return syms.view(K, N // 2 // S, S).transpose(0, 1).reshape(-1, S).contiguous()


@pytest.mark.parametrize("K,N,S,tile", [(64, 256, 32, 8), (130, 512, 64, 0), (256, 2048, 256, 8)])
def test_split_encode_is_reference_encoder_on_rearranged_symbols(K, N, S, tile):
    x = inputs(K, N, K + N)
    comp, st, off, part, sm, pf, sp = tans_codec.encode(x, QWEN, tile=tile, segment_pairs=S)
    want = oracle.encode(split_syms(x, S), pf.numpy(), sp.numpy())
    for g_, w_ in zip((comp, st, off, part), want):
        assert np.array_equal(g_.numpy(), w_)
    # sign/mantissa keep the unsplit layout
    assert torch.equal(sm, tans_codec.encode(x, QWEN, tile=tile)[4])
    assert st.numel() == K * (N // 2 // S)


def test_split_streams_decode_on_cpu():
    """Each sub-stream decodes on its own (oracle), and the pieces reassemble."""
    K, N, S = 96, 512, 64
    x = inputs(K, N, 5)
    comp, st, off, part, sm, pf, sp = tans_codec.encode(x, QWEN, segment_pairs=S)
    C = N // 2 // S
    tab = tans_codec.build_decode_table(sp.numpy(), pf.numpy())
    # sm [P][K] -> per sub-stream [S][C*K] in segment-major order
    sm_sub = sm.view(C, S, K).permute(1, 0, 2).reshape(S, C * K).contiguous()
    out, ok = oracle.decode(comp, off, st, part, sm_sub, tab, 2 * S)
    assert ok
    rebuilt = torch.from_numpy(out).view(2 * S, C, K).permute(2, 1, 0).reshape(K, N)
    assert torch.equal(rebuilt, x)


def test_split_arguments_checked():
    x = inputs(64, 256, 1)
    with pytest.raises(AssertionError, match="segment_pairs"):
        tans_codec.encode(x, QWEN, segment_pairs=48)


@pytest.mark.gpu
@pytest.mark.parametrize("K,N,S,tile", [(64, 256, 32, 8), (130, 512, 64, 0), (256, 2048, 256, 8),
                                        (1024, 32768, 4096, 8), (96, 4096, 8, 0)])
def test_device_split_encode_matches_host(cuda, K, N, S, tile):
    x = inputs(K, N, K * 3 + N)
    dev = tans_codec.encode(x.to(cuda), QWEN, tile=tile, segment_pairs=S)
    host = tans_codec.encode(x, QWEN, tile=tile, segment_pairs=S)
    for d, h in zip(dev, host):
        assert torch.equal(d.cpu(), h.cpu())


@pytest.mark.gpu
@pytest.mark.parametrize("K,N,S", [(1024, 2048, 256), (4096, 32768, 4096), (256, 131072, 4096),
                                   (96, 256, 8)])
def test_fused_and_decode_on_split_streams(cuda, K, N, S):
    a = inputs(K, N, K + N).to(cuda)
    b = inputs(K, N, K + N + 1).to(cuda)
    ea = tans_codec.encode(a, QWEN, tile=8, segment_pairs=S)
    eb = tans_codec.encode(b, QWEN, tile=8, segment_pairs=S)
    tbl = tans_codec.build_decode_table(ea[6].numpy(), ea[5].numpy()).to(cuda)
    out = fp8_vecadd_fused_tans(ea[0], ea[2], ea[1], ea[3], ea[4], eb[0], eb[2], eb[1], eb[3],
                                eb[4], tbl, N, segment_pairs=S)
    raw = fp8_vecadd_raw(a.reshape(-1), b.reshape(-1)).view(K, N)
    assert torch.equal(out.view(N // 16, K, 16).permute(1, 0, 2).reshape(K, N), raw)
    e0 = tans_codec.encode(a, QWEN, tile=0, segment_pairs=S)
    dec = gpu_tans_decode(e0[0], e0[2], e0[1], e0[3], e0[4], e0[6].to(cuda), e0[5].to(cuda), N,
                          segment_pairs=S)
    assert torch.equal(dec.t(), a)


@pytest.mark.gpu
def test_split_needs_whole_warps_of_streams(cuda):
    x = inputs(40, 256, 2)
    e = tans_codec.encode(x.to(cuda), QWEN, tile=8, segment_pairs=32)
    tbl = tans_codec.build_decode_table(e[6].numpy(), e[5].numpy()).to(cuda)
    with pytest.raises(RuntimeError, match="divisible by 32"):
        fp8_vecadd_fused_tans(e[0], e[2], e[1], e[3], e[4], e[0], e[2], e[1], e[3], e[4], tbl,
                              256, segment_pairs=32)
