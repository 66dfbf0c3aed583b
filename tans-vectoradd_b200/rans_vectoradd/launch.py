"""Multi-GPU launcher: one process per GPU, each decoding its own share.

The vecadd / decode path has no exchange step, so a job of W ranks is W
independent shards: rank r owns the contiguous range of whole 128-stream
encoder blocks given by `shard.block_range`, loads only those bytes (from an
on-disk container, or by slicing tensors already in host memory), runs the
fused kernel on its GPU and keeps its part of the tiled output.  The process
group is used for the start barrier and for reducing times and checks across
ranks, never on the data path.

    torchrun --nproc-per-node 8 -m rans_vectoradd.launch \\
        --a a.safetensors --b b.safetensors [--steps 20]

prints one JSON line (rank 0) with the aggregate uncompressed-equivalent
GB/s, the max-over-ranks time per step and whether every rank's result
matched the raw FP8 add when the raw inputs are given (--raw-a/--raw-b).

Failure handling: the process group is created with a short timeout
(`timeout_s`, default 60 s), so a rank that dies or never arrives turns the
other ranks' next collective into an error instead of a hang.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

from . import container, fp8_vecadd_fused_tans, tans_codec


def init_from_env(backend: str | None = None, timeout_s: float = 60.0):
    """Initialise torch.distributed from torchrun's environment (RANK,
    WORLD_SIZE, LOCAL_RANK, MASTER_ADDR/PORT); one GPU per process.
    Returns (rank, world, device)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cuda = torch.cuda.is_available()
    dev = torch.device("cuda", local) if cuda else torch.device("cpu")
    if cuda:
        torch.cuda.set_device(dev)
    if world > 1 and not dist.is_initialized():
        backend = backend or ("nccl" if cuda else "gloo")
        kw = {"device_id": dev} if backend == "nccl" else {}
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return rank, world, dev


def load_shard(path: str, device, rank: int, world: int):
    """This rank's encoder blocks of one encoded input from a container file:
    (comp, offsets, states, partial, sm) in kernel order, plus metadata."""
    (comp, states, offsets, partial, sm, pf, sp), meta = container.load_encoded(
        path, device, rank=rank, world=world)
    return [comp, offsets, states, partial, sm], pf, sp, meta


def run_sharded_vecadd(a_path: str, b_path: str, device, rank: int, world: int,
                       steps: int = 10, warmup: int = 3):
    """Load this rank's shards of inputs A and B, build the shared decode
    table, run the fused kernel `warmup + steps` times, and return (tiled
    output, per-step ms on this rank, stream range, n_fp8_per_stream)."""
    a, pf, sp, meta = load_shard(a_path, device, rank, world)
    b, pf_b, sp_b, _ = load_shard(b_path, device, rank, world)
    if not (torch.equal(pf, pf_b) and torch.equal(sp, sp_b)):
        raise ValueError("A and B must share one table (encode both with the same exp_freqs)")
    N = int(meta["n_fp8_per_stream"])
    if int(meta["tile"]) != 8:
        raise ValueError("the fused add needs inputs encoded with tile=8")
    table = tans_codec.build_decode_table(sp.numpy(), pf.numpy()).to(device)
    out = None
    for _ in range(warmup):
        out = fp8_vecadd_fused_tans(*a, *b, table, N)
    stream = torch.cuda.current_stream(device)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    t0.record(stream)
    for _ in range(steps):
        out = fp8_vecadd_fused_tans(*a, *b, table, N)
    t1.record(stream)
    torch.cuda.synchronize(device)
    s0, s1 = (int(v) for v in meta["stream_range"].split(":"))
    return out, t0.elapsed_time(t1) / steps, (s0, s1), N


def _max_over_ranks(v: float, world: int, device) -> float:
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--a", required=True, help="container of input A (tile=8)")
    ap.add_argument("--b", required=True, help="container of input B (same table)")
    ap.add_argument("--raw-a", help="optional raw e4m3 bytes of A (.pt, [K, N] uint8) to check")
    ap.add_argument("--raw-b", help="optional raw e4m3 bytes of B")
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--timeout", type=float, default=60.0)
    args = ap.parse_args(argv)
    rank, world, dev = init_from_env(timeout_s=args.timeout)
    try:
        out, ms, (s0, s1), N = run_sharded_vecadd(args.a, args.b, dev, rank, world,
                                                  args.steps, args.warmup)
        ok = True
        if args.raw_a and args.raw_b:
            from . import fp8_vecadd_raw
            xa = torch.load(args.raw_a)[s0:s1].contiguous().to(dev)
            xb = torch.load(args.raw_b)[s0:s1].contiguous().to(dev)
            raw = fp8_vecadd_raw(xa.reshape(-1), xb.reshape(-1)).view(s1 - s0, N)
            ok = torch.equal(out.view(N // 16, s1 - s0, 16).permute(1, 0, 2).reshape(s1 - s0, N),
                             raw)
        ms_max = _max_over_ranks(ms, world, dev)
        elems = torch.tensor([float((s1 - s0) * N)], dtype=torch.float64, device=dev)
        good = torch.tensor([1.0 if ok else 0.0], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(elems)
            dist.all_reduce(good)
        if rank == 0:
            n = float(elems.item())
            print(json.dumps({"launcher": "rans_vectoradd.launch", "ranks": world,
                              "ms_per_step_max": round(ms_max, 4),
                              "gbs_uncompressed_equiv": round(3.0 * n / (ms_max / 1e3) / 1e9, 2),
                              "elements_per_input": int(n),
                              "ranks_bit_exact": int(good.item())}), flush=True)
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
