"""Multi-GPU partitioning of encoded tensors (one process per GPU).

The vecadd/decode path has no exchange step: its streams are independent, so
rank r of W simply owns a contiguous range of whole 128-stream encoder blocks
of every input (compressed bytes, offsets rebased to 0, states, partial
counts, sign/mantissa columns) and writes its own output.  The GEMV stack
shards W by rows and reassembles y with an all-gather; `gather_rows` turns
the gathered [world, batch, rows/world] buffer back into [batch, rows].
"""
from __future__ import annotations

import torch

BLOCK = 128


def block_range(n_streams: int, rank: int, world: int) -> tuple[int, int]:
    """[first, last) encoder blocks owned by `rank`: contiguous, sizes differ by
    at most one block."""
    blocks = (n_streams + BLOCK - 1) // BLOCK
    base, extra = divmod(blocks, world)
    first = rank * base + min(rank, extra)
    return first, first + base + (1 if rank < extra else 0)


def shard_encoded(comp, offsets, states, partial, sm, rank: int, world: int, tile: int = 0):
    """This rank's slice of one encoded input (host or device tensors).

    `sm` is [N/2, K] (tile == 0) or tiled [N/2/tile, K, tile].  Returns
    (comp, offsets, states, partial, sm) for the rank's streams, offsets
    rebased so the slice is a valid encoded input on its own."""
    K = states.numel()
    b0, b1 = block_range(K, rank, world)
    s0, s1 = b0 * BLOCK, min(b1 * BLOCK, K)
    lo, hi = int(offsets[b0]), int(offsets[b1])
    off = (offsets[b0:b1 + 1].to(torch.int64) - lo).to(torch.int32)
    sm_r = sm[:, s0:s1].contiguous()  # stream axis is dim 1 in both layouts
    return comp[lo:hi].contiguous(), off.contiguous(), states[s0:s1].contiguous(), \
        partial[s0:s1].contiguous(), sm_r


def gather_rows(gathered: torch.Tensor) -> torch.Tensor:
    """[world, batch, rows_per_rank] (the output of all_gather_into_tensor of
    each rank's [batch, rows_per_rank] y shard into a [world * batch,
    rows_per_rank] buffer, viewed as 3-D) -> [batch, world * rows_per_rank]."""
    w, b, r = gathered.shape
    return gathered.permute(1, 0, 2).reshape(b, w * r)
