"""The allocation-free decode entry point, tans_b200_decode_noalloc.

It serves callers that cannot allocate device memory themselves (a runtime
that only hands out buffers from a pre-sized pool, or a host-language binding
without a device allocator): they pass inputs and outputs only, and the decode
table lives in a fixed 16 KiB device array inside the library.  Here it is
called through the C ABI and compared byte for byte with the regular decode
path (gpu_tans_decode), on two calls in a row that use different tables, so a
stale table from the first call would show up in the second.

This file sorts last so that a run stopping at the first failure has already
run every other test.
"""
from __future__ import annotations

import pytest
import torch

from rans_vectoradd import QWEN3_14B_FP8_EXP, gpu_tans_decode, random_fp8_bytes, tans_codec
from rans_vectoradd._lib import LIB


def _decode_noalloc(dev, comp, off, st, part, sm, sp, pf, N, status):
    K = st.numel()
    out = torch.empty((N, K), dtype=torch.uint8, device=dev)
    rc = LIB.tans_b200_decode_noalloc(
        comp.data_ptr(), comp.numel(), off.data_ptr(), st.data_ptr(), part.data_ptr(),
        sm.data_ptr(), sp.data_ptr(), pf.data_ptr(), pf.numel(), out.data_ptr(), K, N,
        status.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
    assert rc == 0, LIB.tans_b200_last_error().decode()
    return out


@pytest.mark.gpu
def test_noalloc_decode_matches_regular_decode_twice(cuda):
    flat = tuple([1.0] * 16)  # a second exponent profile, so the two tables differ
    cases = [(21, 1000, 256, QWEN3_14B_FP8_EXP), (22, 333, 1024, flat)]
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    for seed, K, N, profile in cases:
        gen = torch.Generator().manual_seed(seed)
        fp8 = random_fp8_bytes(K * N, device="cpu", generator=gen,
                               exp_probs=profile).reshape(K, N)
        comp, st, off, part, sm, pf, sp = tans_codec.encode(
            fp8, torch.tensor(profile, dtype=torch.float64))
        args = [t.to(cuda) for t in (comp, off, st, part, sm, sp, pf)]
        ref = gpu_tans_decode(*args, N)
        out = _decode_noalloc(cuda, *args, N, status)
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
        assert torch.equal(out.cpu().t(), fp8)
        assert int(status.item()) == 0


def test_noalloc_rejects_alphabet_beyond_scratch():
    rc = LIB.tans_b200_decode_noalloc(None, 4, None, None, None, None, None, None, 257, None,
                                      1, 2, None, None)
    assert rc == 1
    assert "exceeds the scratch table" in LIB.tans_b200_last_error().decode()
