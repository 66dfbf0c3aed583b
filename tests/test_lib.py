"""The C-ABI library: loads, exports every symbol include/tans_b200.h
declares, and rejects bad arguments before touching a device.  CPU only."""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

import pytest
import torch

from rans_vectoradd import _C
from rans_vectoradd._lib import LIB, LIB_PATH, check, version

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "tans_b200.h")


def declared_functions() -> list[str]:
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(tans_b200_\w+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "tans_b200_fp8_vecadd_fused" in names and "tans_b200_decode" in names
    assert len(names) >= 14


def test_library_exports_every_declared_symbol():
    for name in declared_functions():
        assert hasattr(LIB, name), name


def test_exports_with_nm():
    out = subprocess.run(["nm", "-D", "--defined-only", LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (tans_b200_\w+)", out))
    assert set(declared_functions()) <= exported


def test_header_compiles_as_c(tmp_path):
    src = tmp_path / "t.c"
    src.write_text('#include "tans_b200.h"\nint main(void){return TANS_B200_OK;}\n')
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.dirname(HEADER),
                    "-c", str(src), "-o", str(tmp_path / "t.o")], check=True)


def test_version():
    assert "sm_100a" in version()


def test_invalid_sizes_rejected_without_device():
    # size checks happen before any CUDA call
    rc = LIB.tans_b200_fp8_vecadd_raw(None, None, None, 17, None)
    assert rc == 1 and "multiple of 16" in LIB.tans_b200_last_error().decode()
    rc = LIB.tans_b200_fp8_memcpy(None, None, 15, None)
    assert rc == 1
    rc = LIB.tans_b200_decode(None, 4, None, None, None, None, None, None, 4, 3, None, None)
    assert rc == 1 and "even" in LIB.tans_b200_last_error().decode()
    rc = LIB.tans_b200_fp8_vecadd_fused(None, 0, None, None, None, None, None, 0, None, None,
                                        None, None, None, None, 4, 24, None, None)
    assert rc == 1 and "divisible by 16" in LIB.tans_b200_last_error().decode()
    rc = LIB.tans_b200_build_decode_table(None, None, 256, None, None, None)
    assert rc == 1
    with pytest.raises(RuntimeError, match="multiple of 16"):
        check(LIB.tans_b200_fp8_vecadd_raw(None, None, None, 17, None))


def test_zero_length_calls_are_noops():
    assert LIB.tans_b200_fp8_vecadd_raw(None, None, None, 0, None) == 0
    assert LIB.tans_b200_decode(None, 0, None, None, None, None, None, None, 0, 8, None,
                                None) == 0


def test_encoder_handle_lifecycle():
    syms = torch.zeros((3, 10), dtype=torch.uint8)
    f = torch.zeros(256, dtype=torch.int32)
    f[0] = 4096
    sp = torch.zeros(4096, dtype=torch.int32)
    h = ctypes.c_void_p()
    check(LIB.tans_b200_encode(syms.data_ptr(), 3, 10, f.data_ptr(), 256, sp.data_ptr(), 1,
                               ctypes.byref(h)))
    nb, nblk = ctypes.c_int64(), ctypes.c_int64()
    check(LIB.tans_b200_encoded_sizes(h, ctypes.byref(nb), ctypes.byref(nblk)))
    assert nb.value == 512 and nblk.value == 1
    LIB.tans_b200_encoded_free(h)


def test_op_checks_mirror_reference_messages():
    """TORCH_CHECK messages of csrc/vecadd.cu:268-337, csrc/fp8_memcpy.cu:45-49,
    csrc/tans_decode.cu:169-191, raised before any device work."""
    cpu = torch.zeros(32, dtype=torch.uint8)
    with pytest.raises(RuntimeError, match="A must be CUDA"):
        _C.fp8_vecadd_raw(cpu, cpu)
    with pytest.raises(RuntimeError, match="A must be CUDA"):
        _C.fp8_memcpy(cpu)
    with pytest.raises(RuntimeError, match="compressed must be contiguous CUDA uint8"):
        _C.gpu_tans_decode(cpu, cpu, cpu, cpu, cpu, cpu, cpu, 16)
    with pytest.raises(RuntimeError, match="a_comp must be CUDA"):
        _C.fp8_vecadd_fused_tans(*([cpu] * 11), 16)


def test_streams_per_block_env_validation(monkeypatch):
    monkeypatch.setenv("TANS_STREAMS_PER_BLOCK", "3")
    with pytest.raises(RuntimeError, match="one of 1, 2, 4, or 8"):
        _C._streams_per_block_from_env()
    monkeypatch.setenv("TANS_STREAMS_PER_BLOCK", "x")
    with pytest.raises(RuntimeError, match="must be an integer"):
        _C._streams_per_block_from_env()
    monkeypatch.setenv("TANS_STREAMS_PER_BLOCK", "4")
    assert _C._streams_per_block_from_env() == 4


def test_gather_descriptor_matches_header(tmp_path):
    """rans_vectoradd.peer.GatherDesc has the layout of tans_b200_gather."""
    from rans_vectoradd.peer import GatherDesc, layout
    src = tmp_path / "g.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "tans_b200.h"\n'
                   "int main(void) { printf(\"%zu\", sizeof(tans_b200_gather));\n"
                   + "".join(f' printf(" %zu", offsetof(tans_b200_gather, {f}));'
                             for f, _ in GatherDesc._fields_) + " return 0; }\n")
    exe = tmp_path / "g"
    subprocess.run(["gcc", "-std=c11", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)],
                   check=True)
    got = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True,
                                          check=True).stdout.split()]
    assert got == [ctypes.sizeof(GatherDesc)] + [getattr(GatherDesc, f).offset
                                                 for f, _ in GatherDesc._fields_]
    offs, total = layout([1024, 512], 3, 8)
    assert offs[0] >= 32 and all(o % 256 == 0 for o in offs) and total % 256 == 0
    assert offs[1] - offs[0] >= 3 * 1024 * 2 and total - offs[1] >= 3 * 512 * 2


def test_gemv_gather_rejects_bad_descriptors_without_device():
    from rans_vectoradd.peer import GatherDesc
    d = ctypes.c_void_p(16)  # never dereferenced: the checks come first
    args = [d, 4, d, d, d, d, d, d, d, d, 32, 64, 1, 1]
    assert LIB.tans_b200_gemv_gather(*args, None, None, None) == 1
    bad = GatherDesc(2, 2, 16, 64, 0, 16, 16, 16, 16)  # rank outside [0, world)
    assert LIB.tans_b200_gemv_gather(*args, ctypes.addressof(bad), None, None) == 1
    assert "rank 2 of 2" in LIB.tans_b200_last_error().decode()
    odd = GatherDesc(0, 2, 16, 64, 1, 16, 16, 16, 16)  # odd column offset
    assert LIB.tans_b200_gemv_gather(*args, ctypes.addressof(odd), None, None) == 1
