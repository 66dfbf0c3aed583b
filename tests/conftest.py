"""Shared pytest setup.

Markers: `gpu` — needs a CUDA device (run with -m gpu on a B200).  Everything
else runs on CPU.  The product package lives in tans-vectoradd_b200/ and the
test-only oracle in oracle/; both are put on sys.path here.
"""
from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "tans-vectoradd_b200")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (PKG, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden_digests():
    import json
    with open(os.path.join(GOLDEN, "digests.json")) as f:
        return json.load(f)["cases"]


@pytest.fixture(scope="session")
def ref_ext():
    """The reference's own compiled _C (oracle/_ref), or skip."""
    import oracle
    ext = oracle.load_ref_ext()
    if ext is None:
        pytest.skip("reference extension not built (oracle/build_ref.sh)")
    return ext


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
