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


def test_noalloc_rejects_alphabet_beyond_table_build():
    rc = LIB.tans_b200_decode_noalloc(None, 4, None, None, None, None, None, None, 257, None,
                                      1, 2, None, None)
    assert rc == 1
    assert "alphabet must be 1..256 symbols" in LIB.tans_b200_last_error().decode()


@pytest.mark.gpu
def test_noalloc_decode_allocates_no_device_memory(cuda):
    """The defining property: after a first call (which resolves the scratch
    array's device address), further calls on the current and on a second
    stream leave the device's free memory unchanged."""
    gen = torch.Generator().manual_seed(23)
    K, N = 512, 512
    fp8 = random_fp8_bytes(K * N, device="cpu", generator=gen).reshape(K, N)
    comp, st, off, part, sm, pf, sp = tans_codec.encode(
        fp8, torch.tensor(QWEN3_14B_FP8_EXP, dtype=torch.float64))
    args = [t.to(cuda) for t in (comp, off, st, part, sm, sp, pf)]
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    outs = [torch.empty((N, K), dtype=torch.uint8, device=cuda) for _ in range(2)]
    side = torch.cuda.Stream(cuda)

    def call(out, stream):
        rc = LIB.tans_b200_decode_noalloc(
            args[0].data_ptr(), args[0].numel(), args[1].data_ptr(), args[2].data_ptr(),
            args[3].data_ptr(), args[4].data_ptr(), args[5].data_ptr(), args[6].data_ptr(),
            args[6].numel(), out.data_ptr(), K, N, status.data_ptr(), stream.cuda_stream)
        assert rc == 0, LIB.tans_b200_last_error().decode()

    call(outs[0], torch.cuda.current_stream(cuda))
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(cuda)
    for _ in range(3):
        call(outs[0], torch.cuda.current_stream(cuda))
    torch.cuda.synchronize()
    side.wait_stream(torch.cuda.current_stream(cuda))
    for _ in range(3):
        call(outs[1], side)
    side.synchronize()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(cuda)
    assert free1 == free0
    assert torch.equal(outs[0].cpu().t(), fp8) and torch.equal(outs[1].cpu().t(), fp8)
