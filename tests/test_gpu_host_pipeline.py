"""The fused decode + add on a stream range (tans_b200_fp8_vecadd_fused_range)
and from host memory (tans_b200_fp8_vecadd_fused_host, chunked and pipelined
over CUDA streams): byte-identical to the one-call device path."""
from __future__ import annotations

import ctypes

import pytest
import torch

from rans_vectoradd import QWEN3_14B_FP8_EXP, _C, fp8_vecadd_fused_tans, random_fp8_bytes, tans_codec
from rans_vectoradd._lib import LIB, check

QWEN = torch.tensor(QWEN3_14B_FP8_EXP, dtype=torch.float64)


def fused_inputs(K, N, seed):
    gen = torch.Generator().manual_seed(seed)
    a = random_fp8_bytes(K * N, device="cpu", generator=gen).reshape(K, N)
    b = random_fp8_bytes(K * N, device="cpu", generator=gen).reshape(K, N)
    ea = tans_codec.encode(a, QWEN, tile=8)
    eb = tans_codec.encode(b, QWEN, tile=8)
    tbl = tans_codec.build_decode_table(ea[6].numpy(), ea[5].numpy())
    return (ea[0], ea[2], ea[1], ea[3], ea[4], eb[0], eb[2], eb[1], eb[3], eb[4], tbl)


@pytest.mark.gpu
@pytest.mark.parametrize("K,N,chunk,pin", [(10_000, 256, 0, True), (10_000, 256, 1000, False),
                                           (129, 2048, 128, True), (65_536, 512, 4096, True)])
def test_host_pipeline_equals_device_call(cuda, K, N, chunk, pin):
    args = fused_inputs(K, N, K + N)
    want = fp8_vecadd_fused_tans(*[t.to(cuda) for t in args], N).cpu()
    host = [t.pin_memory() if pin else t for t in args]
    out = _C.fp8_vecadd_fused_tans_host(*host, N, device=cuda, chunk_streams=chunk)
    torch.cuda.current_stream(cuda).synchronize()
    assert torch.equal(out, want)
    assert _C.data_status(cuda) == 0


@pytest.mark.gpu
def test_range_call_writes_only_its_streams(cuda):
    K, N = 1000, 128
    d = [t.to(cuda) for t in fused_inputs(K, N, 5)]
    full = fp8_vecadd_fused_tans(*d, N)
    out = torch.full_like(full, 0xA5)
    s0, s1 = 256, 700
    ptrs = [t.data_ptr() for t in d]
    check(LIB.tans_b200_fp8_vecadd_fused_range(
        ptrs[0], d[0].numel(), ptrs[1], ptrs[2], ptrs[3], ptrs[4],
        ptrs[5], d[5].numel(), ptrs[6], ptrs[7], ptrs[8], ptrs[9],
        ptrs[10], out.data_ptr(), K, N, s0, s1, None,
        torch.cuda.current_stream(cuda).cuda_stream))
    o = out.view(N // 16, K, 16).cpu()
    f = full.view(N // 16, K, 16).cpu()
    assert torch.equal(o[:, s0:s1], f[:, s0:s1])
    assert (o[:, :s0] == 0xA5).all() and (o[:, s1:] == 0xA5).all()


def test_range_and_host_entry_argument_checks():
    """Argument errors are reported before any CUDA call (CPU only)."""
    nul = [None, 0, None, None, None, None] * 2 + [None, None]
    rc = LIB.tans_b200_fp8_vecadd_fused_range(*nul, 1000, 128, 100, 200, None, None)
    assert rc == 1 and b"128-stream block" in LIB.tans_b200_last_error()
    rc = LIB.tans_b200_fp8_vecadd_fused_range(*nul, 1000, 128, 0, 1001, None, None)
    assert rc == 1
    K, N = 300, 32
    a_off = torch.tensor([0, 1024, 512, 1536], dtype=torch.int32)  # not monotone
    ok_off = torch.tensor([0, 512, 1024, 1536], dtype=torch.int32)
    comp = torch.zeros(1536, dtype=torch.uint8)
    st = torch.zeros(K, dtype=torch.int16)
    part = torch.zeros(K, dtype=torch.uint8)
    sm = torch.zeros(K * N // 2, dtype=torch.uint8)
    tbl = torch.zeros(4096, dtype=torch.int32)
    out = torch.zeros(K * N, dtype=torch.uint8)
    need = ctypes.c_int64()
    check(LIB.tans_b200_fp8_vecadd_fused_host_workspace_bytes(K, N, 1536, 1536, ctypes.byref(need)))
    assert need.value >= 2 * 1536 + K * N
    rc = LIB.tans_b200_fp8_vecadd_fused_host(
        comp.data_ptr(), 1536, a_off.data_ptr(), st.data_ptr(), part.data_ptr(), sm.data_ptr(),
        comp.data_ptr(), 1536, ok_off.data_ptr(), st.data_ptr(), part.data_ptr(), sm.data_ptr(),
        tbl.data_ptr(), out.data_ptr(), K, N, 0, 256, need.value, None, None)
    assert rc == 1 and b"malformed block offsets" in LIB.tans_b200_last_error()
    rc = LIB.tans_b200_fp8_vecadd_fused_host(
        comp.data_ptr(), 1536, ok_off.data_ptr(), st.data_ptr(), part.data_ptr(), sm.data_ptr(),
        comp.data_ptr(), 1536, ok_off.data_ptr(), st.data_ptr(), part.data_ptr(), sm.data_ptr(),
        tbl.data_ptr(), out.data_ptr(), K, N, 0, 256, need.value - 1, None, None)
    assert rc == 1 and b"workspace" in LIB.tans_b200_last_error()
