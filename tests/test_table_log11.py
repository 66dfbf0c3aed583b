"""table_log = 11 (a 2048-entry table): a labelled extra beside the
reference's L = 4096 (rans_vectoradd/tans_codec.py:24-25 fixes L; the
reference has no other size, so nothing of the reference pins these bytes).

The L = 2048 path is checked by properties that do not depend on the size:
the host and numpy table builders agree, the library build for it exports
what the header declares, CPU encode -> oracle decode (run with L = 2048)
returns the input, and on the GPU decode returns the input, the fused add
equals the uncompressed add bit for bit, and the device encoder writes the
host encoder's bytes.
"""
from __future__ import annotations

import re
import subprocess

import numpy as np
import pytest
import torch

import oracle
from rans_vectoradd import _C, tans_codec
from rans_vectoradd._lib import LIB_PATH_L11, lib_for_table

from test_lib import declared_functions


def normal_fp8(K: int, N: int, seed: int, scale: float = 0.5) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(K, N, generator=g) * scale).to(torch.float8_e4m3fn).view(torch.uint8)


def exp_hist(x: torch.Tensor) -> torch.Tensor:
    return torch.bincount(((x >> 3) & 0xF).flatten().long(), minlength=16).float() + 1.0


def test_l11_library_loads_and_exports_every_declared_symbol():
    lib = lib_for_table(2048)
    assert lib.tans_b200_table_size() == 2048
    assert lib_for_table(4096).tans_b200_table_size() == 4096
    out = subprocess.run(["nm", "-D", "--defined-only", LIB_PATH_L11], capture_output=True,
                         text=True, check=True).stdout
    assert set(declared_functions()) <= set(re.findall(r"\bT (tans_b200_\w+)", out))
    with pytest.raises(RuntimeError, match="4096 entries"):
        _C.build_decode_table_device(torch.zeros(1024, dtype=torch.int32),
                                     torch.ones(1, dtype=torch.int32), torch.device("cpu"))


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_l11_tables(seed):
    x = normal_fp8(64, 512, seed, scale=[0.5, 4.0, 0.02][seed])
    pf = tans_codec.pair_freqs_from_exponents(exp_hist(x), table_log=11)
    assert int(pf.sum()) == 2048 and (pf >= 0).all()
    spread = tans_codec.build_spread(pf)
    assert spread.size == 2048
    assert np.array_equal(np.bincount(spread, minlength=pf.size), pf)
    py = tans_codec.build_decode_table(spread, pf).numpy()
    host = _C.build_decode_table_device(torch.from_numpy(spread), torch.from_numpy(pf),
                                        torch.device("cpu")).numpy()
    assert np.array_equal(py, host)
    # every state of [L, 2L) is reached from exactly one (slot, bits) pair
    nb = (py >> 8) & 15
    base = (py >> 16) & 0xFFFF
    assert ((base >= 2048) & (base < 4096)).all() and (nb <= 11).all()


@pytest.mark.parametrize("K,N,seed", [(128, 256, 0), (200, 1024, 1), (1, 16, 2)])
def test_l11_encode_round_trip_through_oracle(K, N, seed):
    x = normal_fp8(K, N, seed)
    comp, st, off, part, sm, pf, sp = tans_codec.encode(x, exp_hist(x), tile=0, table_log=11)
    assert sp.numel() == 2048
    table = tans_codec.build_decode_table(sp.numpy(), pf.numpy()).numpy()
    out, ok = oracle.decode(comp.numpy(), off.numpy(), st.numpy(), part.numpy(), sm.numpy(),
                            table, N)
    assert ok and np.array_equal(out.T, x.numpy())
    # the L = 4096 parity path on the same input is untouched (and smaller or equal)
    comp12 = tans_codec.encode(x, exp_hist(x), tile=0)[0]
    assert comp12.numel() <= comp.numel() + 4 * 128 * ((K + 127) // 128)


@pytest.mark.gpu
@pytest.mark.parametrize("K,N", [(256, 1024), (1000, 4096)])
def test_l11_gpu_decode_and_fused_add(K, N):
    dev = torch.device("cuda", 0)
    x, y = normal_fp8(K, N, 5), normal_fp8(K, N, 6, scale=2.0)
    hist = exp_hist(torch.cat([x, y]))
    a = tans_codec.encode(x, hist, tile=8, table_log=11)
    b = tans_codec.encode(y, hist, tile=8, table_log=11)
    assert torch.equal(a[6], b[6]) and a[6].numel() == 2048
    tbl = tans_codec.build_decode_table(a[6].numpy(), a[5].numpy()).to(dev)
    _C.data_status(dev)
    def parts(e):  # encode's (comp, states, offsets, partial, sm) in the ops' order
        return [e[i].to(dev) for i in (0, 2, 1, 3, 4)]
    fused = _C.fp8_vecadd_fused_tans(*parts(a), *parts(b), tbl, N)
    raw = _C.fp8_vecadd_raw(x.T.contiguous().view(-1).to(dev), y.T.contiguous().view(-1).to(dev))
    want = raw.view(N // 16, 16, K).permute(0, 2, 1).reshape(-1)
    assert torch.equal(fused, want)
    d = tans_codec.encode(x, hist, tile=0, table_log=11)
    out = _C.gpu_tans_decode(*parts(d), d[6].to(dev), d[5].to(dev), N)
    assert torch.equal(out.cpu(), x.T.contiguous())
    assert _C.data_status(dev) == 0


@pytest.mark.gpu
def test_l11_device_encoder_matches_host():
    dev = torch.device("cuda", 0)
    x = normal_fp8(384, 2048, 9)
    host = tans_codec.encode(x, exp_hist(x), tile=8, table_log=11)
    devc = tans_codec.encode(x.to(dev), exp_hist(x), tile=8, table_log=11)
    for h, d in zip(host[:5], devc[:5]):
        assert d.is_cuda and torch.equal(h, d.cpu())
