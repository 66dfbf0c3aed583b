"""Multi-GPU launcher (rans_vectoradd.launch): failure handling of the
process group on CPU (gloo, two ranks), and the sharded fused add from
container files on the GPU (one rank in-process; two ranks under torchrun
when two GPUs are present)."""
from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
import time

import pytest
import torch
import torch.multiprocessing as mp

from rans_vectoradd import QWEN3_14B_FP8_EXP, container, fp8_vecadd_raw, launch, random_fp8_bytes, tans_codec

QWEN = torch.tensor(QWEN3_14B_FP8_EXP, dtype=torch.float64)
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank), CUDA_VISIBLE_DEVICES="")
    import torch.distributed as dist
    launch.init_from_env(backend="gloo", timeout_s=10.0)
    if rank == 1:
        os._exit(3)  # dies between steps, with nothing in flight
    t0 = time.time()
    try:
        dist.barrier()
        q.put(("no error", time.time() - t0))
    except Exception as e:  # the survivor learns of it from the collective
        q.put((type(e).__name__, time.time() - t0))


def test_dead_rank_surfaces_as_an_error_not_a_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    assert all(p.exitcode is not None for p in procs), "a rank hung"
    kind, waited = q.get(timeout=5)
    assert kind != "no error" and waited < 60


def _containers(tmp_path, K=512, N=256, seed=3):
    g = torch.Generator().manual_seed(seed)
    a = random_fp8_bytes(K * N, device="cpu", generator=g).reshape(K, N)
    b = random_fp8_bytes(K * N, device="cpu", generator=g).reshape(K, N)
    pa, pb = str(tmp_path / "a.safetensors"), str(tmp_path / "b.safetensors")
    container.save_encoded(pa, tans_codec.encode(a, QWEN, tile=8), N, tile=8)
    container.save_encoded(pb, tans_codec.encode(b, QWEN, tile=8), N, tile=8)
    ra, rb = str(tmp_path / "a.pt"), str(tmp_path / "b.pt")
    torch.save(a, ra)
    torch.save(b, rb)
    return a, b, pa, pb, ra, rb


@pytest.mark.gpu
def test_launcher_single_rank(cuda, tmp_path):
    a, b, pa, pb, _, _ = _containers(tmp_path)
    K, N = a.shape
    out, ms, (s0, s1), n = launch.run_sharded_vecadd(pa, pb, cuda, 0, 1, steps=2, warmup=1)
    assert (s0, s1, n) == (0, K, N) and ms > 0
    raw = fp8_vecadd_raw(a.reshape(-1).to(cuda), b.reshape(-1).to(cuda)).view(K, N)
    assert torch.equal(out.view(N // 16, K, 16).permute(1, 0, 2).reshape(K, N), raw)


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_launcher_two_ranks(tmp_path):
    _, _, pa, pb, ra, rb = _containers(tmp_path, K=1024)
    env = dict(os.environ, PYTHONPATH=os.pathsep.join(
        [os.path.join(ROOT, "tans-vectoradd_b200"), os.environ.get("PYTHONPATH", "")]))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           "-m", "rans_vectoradd.launch", "--a", pa, "--b", pb, "--raw-a", ra, "--raw-b", rb,
           "--steps", "2", "--warmup", "1", "--timeout", "60"]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads([l for l in r.stdout.splitlines() if l.startswith("{")][-1])
    assert line["ranks"] == 2 and line["ranks_bit_exact"] == 2
    assert line["elements_per_input"] == 1024 * 256


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_gather_stack_two_ranks():
    """Fused peer all-gather of a row-sharded GEMV stack == GEMV + NCCL
    all-gather, bit for bit, eagerly and over CUDA-graph replays."""
    env = dict(os.environ, PYTHONPATH=os.pathsep.join(
        [os.path.join(ROOT, "tans-vectoradd_b200"), os.environ.get("PYTHONPATH", "")]))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "peer_gather_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads([l for l in r.stdout.splitlines() if l.startswith("{")][-1])
    assert line == {"world": 2, "exact": True, "replay_exact": True, "status_clean": True}
