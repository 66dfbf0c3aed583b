"""Rank program for test_peer_gather (run under torchrun, one rank per GPU).

A two-layer up/down GEMV stack, rows sharded over the ranks, run two ways:
plain GEMV + NCCL all-gather (the established path) and the fused peer
gather (tans_b200_gemv_gather: the GEMV epilogue stores its shard into every
rank's symmetric-memory buffer, the next GEMV waits on the peers' flags).
The gathered activations must be identical after every layer, also over
repeated replays of a CUDA graph of the fused forward.  Rank 0 prints one
JSON line.
"""
from __future__ import annotations

import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

from rans_vectoradd import _C, shard, tans_gemv
from rans_vectoradd.peer import PeerGather


def weight(rows, cols, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    w8, s = tans_gemv.quantize_rows(torch.randn(rows, cols, device=dev, generator=g) * 0.02)
    return tans_gemv.encode_weight(w8, s).to(dev)


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    F, H, B, layers = 1024 * world, 512 * world, 3, 2
    fr, hr = F // world, H // world
    ups = [weight(fr, H, 100 * l + rank, dev) for l in range(layers)]
    downs = [weight(hr, F, 100 * l + 50 + rank, dev) for l in range(layers)]
    x0 = torch.randn(B, H, device=dev, generator=torch.Generator(device=dev).manual_seed(3))
    x0 = x0.to(torch.bfloat16)

    def gather(y, full):
        g = torch.empty((world * B, full // world), dtype=torch.bfloat16, device=dev)
        dist.all_gather_into_tensor(g, y.contiguous())
        return shard.gather_rows(g.view(world, B, full // world))

    def forward_nccl():
        outs, x = [], x0
        for up, down in zip(ups, downs):
            h = gather(tans_gemv.gemv(up, x), F)
            x = gather(tans_gemv.gemv(down, h), H)
            outs += [h.clone(), x.clone()]
        return outs

    pg = PeerGather([F, H], B, dev)

    def forward_fused(record):
        outs, x = [], x0
        for up, down in zip(ups, downs):
            h = tans_gemv.gemv_gather(up, x, pg, 0, rank * fr)
            x = tans_gemv.gemv_gather(down, h, pg, 1, rank * hr)
            if record:
                # A gathered buffer is ordered only against the next GEMV that
                # reads it: a faster peer's next up-GEMV may already store
                # into this rank's views[0].  Copy both buffers and hold every
                # rank at a barrier before anyone issues the next layer.
                torch.cuda.synchronize()
                outs += [h.clone(), x.clone()]
                torch.cuda.synchronize()
                dist.barrier()
        return outs

    _C.data_status(dev)
    want = forward_nccl()
    got = forward_fused(True)
    bits = lambda t: t.view(torch.int16)  # noqa: E731  (bit patterns: NaN-safe, exact)
    exact = all(torch.equal(bits(a), bits(b)) for a, b in zip(got, want))
    # the same forward as a CUDA graph, replayed: flags and counters live in
    # device memory, so every replay waits for the right gathers
    for _ in range(2):
        forward_fused(False)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            forward_fused(False)
    torch.cuda.current_stream(dev).wait_stream(side)
    for _ in range(5):
        graph.replay()
    torch.cuda.synchronize()
    replay_exact = torch.equal(bits(pg.views[1]), bits(want[-1]))
    status = _C.data_status(dev)
    del graph
    pg.close()
    t = torch.tensor([float(exact), float(replay_exact), float(status == 0)], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    if rank == 0:
        print(json.dumps({"world": world, "exact": bool(t[0]), "replay_exact": bool(t[1]),
                          "status_clean": bool(t[2])}), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
