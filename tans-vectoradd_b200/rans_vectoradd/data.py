"""Synthetic FP8 E4M3 inputs.

Content matters here: a compressed path's effective bandwidth depends on the
exponent entropy of its inputs, so uniform random bytes (incompressible)
would understate it.  Two sources:

* ``random_fp8_bytes`` — exponents drawn from a 16-bin profile (default: the
  reference's Qwen3-14B-FP8 aggregate, rans_vectoradd/data.py:21-38), sign and
  mantissa uniform.  It consumes the torch RNG exactly as the reference's
  generator does (rans_vectoradd/data.py:41-69: one torch.rand(n) for the
  exponent, one torch.randint(0, 16, (n,), uint8) for sign+mantissa), so a
  seeded call reproduces the reference's bytes.
* ``normal_fp8_bytes`` — values ~ N(0, 1) scaled by 448/max|x| and cast to
  e4m3: the generator of the benchmark configurations (exponent entropy about
  2.54 bits).
"""
from __future__ import annotations

import torch

# Exponent histogram of the FP8 linear weights of Qwen3-14B-FP8 (280 tensors,
# 13.2 GB), entropy 2.787 bits: the reference's encoding source.
QWEN3_14B_FP8_EXP: tuple[float, ...] = (
    0.0005, 0.0005, 0.0009, 0.0018, 0.0034, 0.0062, 0.0104, 0.0167,
    0.0283, 0.0480, 0.0838, 0.1502, 0.2417, 0.2715, 0.1273, 0.0088,
)


def random_fp8_bytes(
    n: int,
    *,
    exp_probs: tuple[float, ...] = QWEN3_14B_FP8_EXP,
    device: str | torch.device = "cuda",
    generator: torch.Generator | None = None,
) -> torch.Tensor:
    """n e4m3 bytes: exponent by inverse CDF of `exp_probs`, sign+mantissa
    uniform over 16 values.  uint8 tensor on `device`."""
    w = torch.tensor(exp_probs, dtype=torch.float32, device=device)
    cdf = torch.cumsum(w / w.sum(), dim=0)
    u = torch.rand(n, device=device, generator=generator)
    exponent = torch.searchsorted(cdf, u).clamp_max_(15).to(torch.uint8)
    sm = torch.randint(0, 16, (n,), dtype=torch.uint8, device=device, generator=generator)
    return ((sm & 8) << 4) | (exponent << 3) | (sm & 7)


def normal_fp8_bytes(
    n: int,
    *,
    device: str | torch.device = "cpu",
    generator: torch.Generator | None = None,
) -> torch.Tensor:
    """n e4m3 bytes of x ~ N(0, 1) scaled so max|x| maps to 448."""
    x = torch.randn(n, device=device, generator=generator)
    x = x * (448.0 / x.abs().max())
    return x.to(torch.float8_e4m3fn).view(torch.uint8)


def exponent_histogram(*fp8: torch.Tensor) -> torch.Tensor:
    """16-bin int64 exponent histogram over all given e4m3 byte tensors."""
    hist = torch.zeros(16, dtype=torch.int64, device=fp8[0].device)
    for t in fp8:
        hist += torch.bincount(((t.reshape(-1) >> 3) & 15).long(), minlength=16)
    return hist
