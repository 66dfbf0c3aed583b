"""Build libtans_b200.so (the C-ABI library) in-tree, for sm_100a only.

    python tans-vectoradd_b200/build.py [--force] [--verbose]

Sources: csrc/kernels.cu (decode/add/GEMV kernels + their entry points),
csrc/encode.cu (device slab encoder), csrc/pipeline.cu (host-memory
pipelined fused add) and csrc/host.cpp (CPU encoder, host table builders,
FP8 splitter, errors).
Output: rans_vectoradd/libtans_b200.so next to the Python package that loads
it, so the built file travels with the source tree, and the same sources
built with a 2048-entry table (-DTANS_B200_TABLE_SIZE=2048, table_log 11, a
labelled extra beside the reference's 4096) as rans_vectoradd/libtans_b200_l11.so.
No torch headers are involved; the libraries depend only on the CUDA runtime
and OpenMP.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
OUT = os.path.join(HERE, "rans_vectoradd", "libtans_b200.so")
OUT_L11 = os.path.join(HERE, "rans_vectoradd", "libtans_b200_l11.so")
VARIANTS = [(OUT, []), (OUT_L11, ["-DTANS_B200_TABLE_SIZE=2048"])]
CU_SOURCES = [os.path.join(CSRC, "kernels.cu"), os.path.join(CSRC, "encode.cu"),
              os.path.join(CSRC, "pipeline.cu")]
HOST_SOURCE = os.path.join(CSRC, "host.cpp")
SOURCES = CU_SOURCES + [HOST_SOURCE, os.path.join(INCLUDE, "tans_b200.h"),
                        os.path.join(CSRC, "internal.h")]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def cuda_home() -> str:
    for cand in (os.environ.get("CUDA_HOME"), "/usr/local/cuda"):
        if cand and os.path.exists(os.path.join(cand, "bin", "nvcc")):
            return cand
    nvcc = shutil.which("nvcc")
    if nvcc:
        return os.path.dirname(os.path.dirname(nvcc))
    raise RuntimeError("nvcc not found: set CUDA_HOME")


def up_to_date(out: str = OUT) -> bool:
    if not os.path.exists(out):
        return False
    t = os.path.getmtime(out)
    return all(os.path.getmtime(s) <= t for s in SOURCES + [__file__])


def build(force: bool = False, verbose: bool = False) -> str:
    """Build every library variant that is missing or older than its sources
    (compiles run in parallel); returns the path of the L = 4096 library."""
    todo = [(out, defs) for out, defs in VARIANTS if force or not up_to_date(out)]
    if not todo:
        return OUT
    cuda = cuda_home()
    nvcc = os.path.join(cuda, "bin", "nvcc")
    # the system g++ carries OpenMP; some images point CXX at a compiler without it
    cxx = shutil.which("g++") or "g++"
    with tempfile.TemporaryDirectory() as tmp:
        cmds, links = [], []
        for vi, (out, defs) in enumerate(todo):
            d = os.path.join(tmp, str(vi))
            os.makedirs(d)
            cu_objs = [os.path.join(d, os.path.basename(s) + ".o") for s in CU_SOURCES]
            h_obj = os.path.join(d, "host.o")
            cmds += [
                [nvcc, "-c", src, "-o", obj, *ARCH, *defs, "-O3", "-lineinfo", "-std=c++17",
                 "-Xcompiler", "-fPIC", "-ccbin", cxx, "-Xptxas", "-v" if verbose else "-O3"]
                for src, obj in zip(CU_SOURCES, cu_objs)
            ] + [
                [cxx, "-c", HOST_SOURCE, "-o", h_obj, *defs, "-O3", "-fPIC", "-fopenmp",
                 "-std=c++17", "-Wall", "-Wextra"],
            ]
            tmp_out = os.path.join(d, os.path.basename(out))
            links.append(([nvcc, "-shared", *ARCH, "-ccbin", cxx, *cu_objs, h_obj, "-o", tmp_out,
                           "-Xcompiler", "-fopenmp", "-lgomp", "-cudart", "shared"], tmp_out, out))
        procs = [subprocess.Popen(c, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
                 for c in cmds]
        failed = None
        for cmd, p in zip(cmds, procs):
            out_txt, _ = p.communicate()
            if verbose or p.returncode:
                sys.stderr.write(out_txt)
            if p.returncode and failed is None:
                failed = cmd
        if failed:
            raise RuntimeError(f"build failed: {' '.join(failed)}")
        for link, tmp_out, out in links:
            r = subprocess.run(link, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
            if r.returncode:
                sys.stderr.write(r.stdout)
                raise RuntimeError("link failed")
            shutil.move(tmp_out, out)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
