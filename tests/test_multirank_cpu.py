"""Multi-rank host logic on CPU with gloo (world size 2): per-rank stream
shards decode to exactly the rank's part of the full result, and the GEMV
stack's all-gather reassembly puts every row back in place."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from rans_vectoradd import QWEN3_14B_FP8_EXP, random_fp8_bytes, shard, tans_codec


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, K, N, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        gen = torch.Generator().manual_seed(5)
        fp8 = random_fp8_bytes(K * N, device="cpu", generator=gen).reshape(K, N)
        prof = torch.tensor(QWEN3_14B_FP8_EXP, dtype=torch.float64)
        comp, st, off, part, sm, pf, sp = tans_codec.encode(fp8, prof)
        tab = tans_codec.build_decode_table(sp.numpy(), pf.numpy())
        c, o, s, p, m = shard.shard_encoded(comp, off, st, part, sm, rank, world)
        out, ok = oracle.decode(c, o, s, p, m, tab, N)  # [N, K_rank]
        b0, b1 = shard.block_range(K, rank, world)
        mine = fp8[b0 * 128:min(b1 * 128, K)]
        good = torch.tensor([int(ok and np.array_equal(out.T, mine.numpy()))])
        dist.all_reduce(good)  # both ranks must decode their shard exactly
        # max-over-ranks timing reduction as bench.py does it
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        # GEMV stack: row shards gathered back into [batch, rows]
        B, rows = 3, 8
        y = torch.arange(B * rows, dtype=torch.float32).reshape(B, rows)
        mine_y = y[:, rank * rows // world:(rank + 1) * rows // world].contiguous()
        g = torch.empty((world * B, rows // world))
        dist.all_gather_into_tensor(g, mine_y)
        same = torch.equal(shard.gather_rows(g.view(world, B, rows // world)), y)
        if rank == 0:
            q.put((int(good.item()), float(t.item()), same))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("K,N", [(300, 64), (256, 128)])
def test_sharded_decode_and_gather_two_ranks(K, N):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, K, N, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    good, tmax, same = q.get(timeout=5)
    assert good == 2 and tmax == 2.0 and same


def test_block_range_partitions_everything():
    for K in (1, 127, 128, 1000, 65536):
        for world in (1, 2, 3, 8):
            spans = [shard.block_range(K, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == (K + 127) // 128
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
