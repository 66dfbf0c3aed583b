"""Generate the golden fixtures in tests/golden/ from the REFERENCE itself.

Run in the build container, where the reference sources are mounted and its
extension has been built from them into oracle/_ref (oracle/build_ref.sh):

    python tests/golden/make_golden.py [REFERENCE_ROOT]

It imports the reference's own Python codec (rans_vectoradd/tans_codec.py,
rans_vectoradd/data.py) together with its compiled `_C`
(csrc/tans_codec.cpp), runs the cases of the reference's own test scripts
(test_gpu_decode_tans.py:69-74, test_vecadd_tans.py:76-80) plus the
benchmark generator of the cfg0 configuration (x, y ~ N(0,1) seed 0, scaled
by 448/max|.|, cast to e4m3), and writes:

  codec_small.npz   full inputs and outputs of the smallest decode case
  tables.npz        pair freqs / spread / decode table (Qwen profile, cfg0)
  digests.json      sha256 of inputs and encoder outputs for every case

Nothing under tests/ reads the reference at test time; only these files.
"""
from __future__ import annotations

import hashlib
import importlib
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def sha(t) -> str:
    a = t.numpy() if hasattr(t, "numpy") else np.asarray(t)
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def load_reference(root: str):
    sys.path.insert(0, REPO)
    import oracle

    ext = oracle.load_ref_ext()
    if ext is None:
        raise SystemExit("reference extension missing: run oracle/build_ref.sh first")
    pkg = types.ModuleType("rans_vectoradd")
    pkg.__path__ = [os.path.join(root, "rans_vectoradd")]
    sys.modules["rans_vectoradd"] = pkg
    sys.modules["rans_vectoradd._C"] = ext
    tc = importlib.import_module("rans_vectoradd.tans_codec")
    data = importlib.import_module("rans_vectoradd.data")
    return tc, data


def encode_case(tc, fp8, exp_freqs, tile):
    comp, st, off, part, sm, pf, sp = tc.encode(fp8, exp_freqs, tile=tile)
    tbl = tc.build_decode_table(sp.numpy(), pf.numpy())
    return dict(compressed=comp, states=st, offsets=off, partial=part, sm=sm,
                pair_freqs=pf, spread=sp, table=tbl)


def digest(case: dict) -> dict:
    return {k: sha(v) for k, v in case.items()} | {
        "compressed_bytes": int(case["compressed"].numel()),
        "sm_bytes": int(case["sm"].numel()),
    }


def cfg0_inputs(n: int):
    g = torch.Generator().manual_seed(0)
    out = []
    for _ in range(2):
        v = torch.randn(n, generator=g)
        v = v * (448.0 / v.abs().max())
        out.append(v.to(torch.float8_e4m3fn).view(torch.uint8))
    return out


def main() -> None:
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get(
        "TANS_REFERENCE_ROOT",
        os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "..", "..", "reference"))
    tc, data = load_reference(root)
    qwen = torch.tensor(data.QWEN3_14B_FP8_EXP, dtype=torch.float64)
    digests: dict = {"torch": torch.__version__, "numpy": np.__version__, "cases": {}}

    # test_gpu_decode_tans.py:17-25,69-74 — seed 42, Qwen profile, tile=0
    for K, N in [(128, 128), (1024, 128), (10_000, 128), (100_000, 128)]:
        torch.manual_seed(42)
        fp8 = data.random_fp8_bytes(K * N, device="cpu").reshape(K, N)
        case = encode_case(tc, fp8, qwen, tile=0)
        digests["cases"][f"decode_K{K}_N{N}"] = {"input": sha(fp8), "K": K, "N": N, "seed": 42,
                                                 "tile": 0} | digest(case)
        if K == 128:
            np.savez_compressed(
                os.path.join(HERE, "codec_small.npz"), fp8=fp8.numpy(),
                **{k: v.numpy() for k, v in case.items()})

    # test_vecadd_tans.py:30-38,76-80 — seed 0, two inputs, tile=8
    for K, N in [(1024, 128), (10_000, 256), (1024, 1024)]:
        torch.manual_seed(0)
        a = data.random_fp8_bytes(K * N, device="cpu").reshape(K, N)
        b = data.random_fp8_bytes(K * N, device="cpu").reshape(K, N)
        ca = encode_case(tc, a, qwen, tile=8)
        cb = encode_case(tc, b, qwen, tile=8)
        digests["cases"][f"fused_K{K}_N{N}"] = {
            "K": K, "N": N, "seed": 0, "tile": 8, "input_a": sha(a), "input_b": sha(b),
            "a": digest(ca), "b": digest(cb)}

    # cfg0 generator: n = 2^24 per input, N = 8192 fp8 per stream, tile=8,
    # one table from the exponent histogram of x and y combined.
    n, N = 1 << 24, 8192
    x, y = cfg0_inputs(n)
    hist = torch.bincount(torch.cat([(x >> 3) & 15, (y >> 3) & 15]).long(), minlength=16)
    ex = encode_case(tc, x.reshape(n // N, N), hist.double(), tile=8)
    ey = encode_case(tc, y.reshape(n // N, N), hist.double(), tile=8)
    digests["cases"]["cfg0"] = {
        "n": n, "N": N, "K": n // N, "seed": 0, "tile": 8, "input_x": sha(x), "input_y": sha(y),
        "exp_hist": hist.tolist(), "x": digest(ex), "y": digest(ey)}

    # tables for the two frequency sources
    torch.manual_seed(42)
    q = encode_case(tc, data.random_fp8_bytes(128 * 128, device="cpu").reshape(128, 128), qwen, 0)
    np.savez_compressed(
        os.path.join(HERE, "tables.npz"),
        qwen_exp=qwen.numpy(), qwen_pair_freqs=q["pair_freqs"].numpy(),
        qwen_spread=q["spread"].numpy(), qwen_table=q["table"].numpy(),
        cfg0_exp_hist=hist.numpy(), cfg0_pair_freqs=ex["pair_freqs"].numpy(),
        cfg0_spread=ex["spread"].numpy(), cfg0_table=ex["table"].numpy(),
        qwen_profile=np.asarray(data.QWEN3_14B_FP8_EXP, np.float64))

    with open(os.path.join(HERE, "digests.json"), "w") as f:
        json.dump(digests, f, indent=1, sort_keys=True)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
