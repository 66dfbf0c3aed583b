"""On-disk container: safetensors layout, round trips, sharded loads equal to
the in-memory partition, and rejection of malformed files (CPU); sharded
device loads decoding bit-exactly (GPU)."""
from __future__ import annotations

import json
import struct

import numpy as np
import pytest
import torch

from rans_vectoradd import QWEN3_14B_FP8_EXP, container, random_fp8_bytes, shard, tans_codec, tans_gemv

QWEN = torch.tensor(QWEN3_14B_FP8_EXP, dtype=torch.float64)


def encoded(K, N, tile, seed=3):
    g = torch.Generator().manual_seed(seed)
    x = random_fp8_bytes(K * N, device="cpu", generator=g).reshape(K, N)
    return x, tans_codec.encode(x, QWEN, tile=tile)


def test_file_is_safetensors_layout(tmp_path):
    _, enc = encoded(300, 64, 8)
    p = str(tmp_path / "a.safetensors")
    container.save_encoded(p, enc, 64, tile=8)
    raw = open(p, "rb").read()
    (hlen,) = struct.unpack("<Q", raw[:8])
    assert (8 + hlen) % 64 == 0
    hdr = json.loads(raw[8:8 + hlen])
    meta = hdr.pop("__metadata__")
    assert meta["format"] == container.FORMAT and meta["n_streams"] == "300"
    assert all(isinstance(v, str) for v in meta.values())
    spans = sorted(v["data_offsets"] for v in hdr.values())
    assert spans[0][0] == 0 and all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    assert spans[-1][1] == len(raw) - 8 - hlen  # fully indexed, no holes
    assert hdr["states"]["dtype"] == "U16" and hdr["offsets"]["dtype"] == "I32"
    assert hdr["sm"]["shape"] == [4, 300, 8]


@pytest.mark.parametrize("tile", [0, 8])
def test_round_trip(tmp_path, tile):
    _, enc = encoded(1000, 128, tile)
    p = str(tmp_path / "e.safetensors")
    container.save_encoded(p, enc, 128, tile=tile)
    got, meta = container.load_encoded(p)
    assert meta["stream_range"] == "0:1000"
    for a, b in zip(got, enc):
        assert a.dtype == b.dtype and torch.equal(a, torch.as_tensor(b))


@pytest.mark.parametrize("world", [2, 3, 8])
def test_sharded_load_equals_partition(tmp_path, world):
    _, enc = encoded(1000, 128, 8)
    comp, states, offsets, partial, sm, pf, sp = enc
    p = str(tmp_path / "e.safetensors")
    container.save_encoded(p, enc, 128, tile=8)
    for rank in range(world):
        got, _ = container.load_encoded(p, rank=rank, world=world)
        want = shard.shard_encoded(comp, offsets, states, partial, sm, rank, world, tile=8)
        for a, b in zip((got[0], got[2], got[1], got[3], got[4]), want):
            assert torch.equal(a, b)


def test_sharded_shards_decode_like_the_whole(tmp_path):
    """Each shard is a valid encoded input on its own (oracle decode)."""
    import oracle
    x, enc = encoded(700, 64, 0)
    p = str(tmp_path / "d.safetensors")
    container.save_encoded(p, enc, 64, tile=0)
    tab = tans_codec.build_decode_table(enc[6].numpy(), enc[5].numpy())
    rows = []
    for rank in range(3):
        (comp, st, off, part, sm, _, _), meta = container.load_encoded(p, rank=rank, world=3)
        out, ok = oracle.decode(comp, off, st, part, sm, tab, 64)
        assert ok
        rows.append(out.T)
    assert np.array_equal(np.concatenate(rows), x.numpy())


def test_gemv_weight_round_trip(tmp_path):
    w = torch.randn(64, 512, generator=torch.Generator().manual_seed(1)) * 0.02
    w8, s = tans_gemv.quantize_rows(w)
    enc = tans_gemv.encode_weight(w8, s, col_splits=2)
    p = str(tmp_path / "w.safetensors")
    container.save_gemv_weight(p, enc)
    got = container.load_gemv_weight(p)
    for name in ("compressed", "offsets", "states", "partial", "sm", "table", "scale"):
        assert torch.equal(getattr(got, name), getattr(enc, name)), name
    assert (got.rows, got.cols, got.col_splits) == (64, 512, 2)


def test_malformed_files_rejected(tmp_path):
    _, enc = encoded(200, 32, 0)
    p = str(tmp_path / "e.safetensors")
    container.save_encoded(p, enc, 32)
    raw = bytearray(open(p, "rb").read())
    bad = tmp_path / "short.safetensors"
    bad.write_bytes(bytes(raw[:4]))
    with pytest.raises(ValueError, match="too short"):
        container.load(str(bad))
    trunc = tmp_path / "trunc.safetensors"
    trunc.write_bytes(bytes(raw[:-10]))
    with pytest.raises(ValueError, match="inconsistent offsets"):
        container.load(str(trunc))
    huge = bytearray(raw)
    huge[:8] = struct.pack("<Q", 1 << 40)
    (tmp_path / "huge.safetensors").write_bytes(bytes(huge))
    with pytest.raises(ValueError, match="exceeds the file"):
        container.load(str(tmp_path / "huge.safetensors"))
    w = torch.randn(16, 64) * 0.02
    container.save_gemv_weight(str(tmp_path / "w.safetensors"),
                               tans_gemv.encode_weight(*tans_gemv.quantize_rows(w)))
    with pytest.raises(ValueError, match="not an encoded-tensor container"):
        container.load_encoded(str(tmp_path / "w.safetensors"))


@pytest.mark.gpu
def test_sharded_device_load_runs_fused(cuda, tmp_path):
    """Rank shards loaded straight to the GPU give the rank's columns of the
    full fused output."""
    from rans_vectoradd import fp8_vecadd_fused_tans
    K, N = 1000, 256
    g = torch.Generator().manual_seed(8)
    a = random_fp8_bytes(K * N, device="cpu", generator=g).reshape(K, N)
    b = random_fp8_bytes(K * N, device="cpu", generator=g).reshape(K, N)
    ea, eb = tans_codec.encode(a, QWEN, tile=8), tans_codec.encode(b, QWEN, tile=8)
    tbl = tans_codec.build_decode_table(ea[6].numpy(), ea[5].numpy()).to(cuda)
    pa, pb = str(tmp_path / "a.safetensors"), str(tmp_path / "b.safetensors")
    container.save_encoded(pa, ea, N, tile=8)
    container.save_encoded(pb, eb, N, tile=8)
    full = fp8_vecadd_fused_tans(*[t.to(cuda) for t in (ea[0], ea[2], ea[1], ea[3], ea[4],
                                                       eb[0], eb[2], eb[1], eb[3], eb[4])],
                                 tbl, N).view(N // 16, K, 16)
    for rank in range(2):
        (ca, sa, oa, qa, ma, _, _), meta = container.load_encoded(pa, cuda, rank, 2)
        (cb, sb, ob, qb, mb, _, _), _ = container.load_encoded(pb, cuda, rank, 2)
        assert ca.is_cuda and ma.is_cuda
        out = fp8_vecadd_fused_tans(ca, oa, sa, qa, ma, cb, ob, sb, qb, mb, tbl, N)
        s0, s1 = (int(v) for v in meta["stream_range"].split(":"))
        assert torch.equal(out.view(N // 16, s1 - s0, 16), full[:, s0:s1])
