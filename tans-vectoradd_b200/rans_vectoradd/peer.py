"""Peer all-gather for row-sharded GEMVs, fused into the GEMV epilogue.

One process per GPU.  Each rank owns a row shard of every weight; after its
GEMV each rank's epilogue stores its shard of y straight into every rank's
gathered buffer over NVLink and raises its flag on every rank; the next
GEMV on each rank waits for all flags before it reads the gathered x
(tans_b200_gemv_gather).  The buffers and flags live in torch symmetric
memory (one allocation per rank, mapped into every peer), so no NCCL call
sits between the layers.

    pg = PeerGather([F, H], batch, device)       # after init_process_group
    tans_gemv.gemv_gather(up, x, pg, 0, rank * F // world)   # y -> pg.views[0]
    tans_gemv.gemv_gather(down, pg.views[0], pg, 1, rank * H // world)

Every rank must issue the same gathers in the same order.  A rank that
stops makes the others' waits run out (TANS_B200_DATA_TIMEOUT in the status
word) instead of hanging them.
"""
from __future__ import annotations

import ctypes
from typing import Sequence

import torch

_ALIGN = 256


class GatherDesc(ctypes.Structure):
    """tans_b200_gather (include/tans_b200.h)."""
    _fields_ = [("rank", ctypes.c_int32), ("world", ctypes.c_int32),
                ("y_peers", ctypes.c_void_p), ("y_ld", ctypes.c_int64),
                ("col0", ctypes.c_int64), ("flag_peers", ctypes.c_void_p),
                ("flags", ctypes.c_void_p), ("seq", ctypes.c_void_p), ("done", ctypes.c_void_p)]


def _round_up(n: int, a: int) -> int:
    return (n + a - 1) // a * a


def layout(widths: Sequence[int], batch: int, world: int) -> tuple[list[int], int]:
    """Byte offsets of the gathered buffers in the per-rank allocation (the
    flag array first) and its total size."""
    off = _round_up(4 * world, _ALIGN)
    offs = []
    for w in widths:
        offs.append(off)
        off += _round_up(batch * w * 2, _ALIGN)
    return offs, off


class PeerGather:
    """Gathered bf16 buffers [batch][width] (one per width) and flags in
    symmetric memory, plus this rank's counters."""

    def __init__(self, widths: Sequence[int], batch: int, device, group=None):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem
        self.group = group if group is not None else dist.group.WORLD
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        self.device = torch.device(device)
        self.widths = [int(w) for w in widths]
        for w in self.widths:
            if w % (2 * self.world) != 0:
                raise ValueError(f"width {w} must split into even shards over {self.world} ranks")
        offs, total = layout(self.widths, batch, self.world)
        self.buf = symm_mem.empty(total, dtype=torch.uint8, device=self.device)
        self.buf.zero_()
        self.hdl = symm_mem.rendezvous(self.buf, self.group.group_name)
        ptrs = [int(p) for p in self.hdl.buffer_ptrs]
        self.flag_peers = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
        self.y_peers = [torch.tensor([p + o for p in ptrs], dtype=torch.int64, device=self.device)
                        for o in offs]
        self.views = [self.buf[o:o + batch * w * 2].view(torch.bfloat16).view(batch, w)
                      for o, w in zip(offs, self.widths)]
        self.flags = self.buf[:4 * self.world]
        self.seq = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.done = torch.zeros(1, dtype=torch.int32, device=self.device)
        # every rank's flags are zero before any rank can raise one
        torch.cuda.synchronize(self.device)
        self.hdl.barrier()

    def descriptor(self, k: int, col0: int) -> GatherDesc:
        """The C descriptor for a gather into buffer k at column col0."""
        return GatherDesc(self.rank, self.world, self.y_peers[k].data_ptr(), self.widths[k],
                          int(col0), self.flag_peers.data_ptr(), self.flags.data_ptr(),
                          self.seq.data_ptr(), self.done.data_ptr())

    def close(self) -> None:
        """Wait until every rank is done with the buffers."""
        torch.cuda.synchronize(self.device)
        self.hdl.barrier()
        torch.cuda.synchronize(self.device)


__all__ = ["GatherDesc", "PeerGather", "layout"]
