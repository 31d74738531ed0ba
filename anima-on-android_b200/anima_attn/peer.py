"""Gather buffers shared by the ranks of one node over NVLink (CUDA IPC).

The head-parallel DiT step gathers every rank's attention output [B, S, H/N, D] into a
[B, S, H, D] tensor on every rank before the output projection.  With GatherBuffers the
attention kernel stores each output block straight into all ranks' buffers
(anima_attn_fwd_gather), and a one-element all-reduce orders the ranks before the buffer is
read, in place of an NCCL all-gather and the transpose after it.

Two buffers alternate (buffer i for the i-th attention of a pair), so a rank never writes a
buffer that a slower rank's output projection is still reading: a rank reaches the next use
of a buffer only after the barrier of the attention in between, which every rank enters
after its own projection of the earlier one.
"""
from __future__ import annotations

import ctypes as ct
from typing import List

import torch

from . import _lib as L


class GatherBuffers:
    """Two [B, S, H, D] buffers of `dtype` on this rank's device, mapped into every rank.

    ``ptrs[i][r]`` is the device address of rank r's buffer i in this process (this rank's
    own buffer included).  Every rank of ``group`` constructs it in the same order; call
    ``close()`` (every rank) before the process group is destroyed."""

    def __init__(self, shape, dtype: torch.dtype, device, group, rank: int, world: int):
        import torch.distributed as dist
        self.rank, self.world = rank, world
        self.bufs = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(2)]
        mine = []
        for b in self.bufs:
            h = (ct.c_char * L.IPC_HANDLE_BYTES)()
            off = ct.c_uint64(0)
            L.check(L.lib.anima_ipc_export(ct.c_void_p(b.data_ptr()), h, ct.byref(off)),
                    "anima_ipc_export")
            mine.append((bytes(h), int(off.value)))
        everyone: List = [None] * world
        dist.all_gather_object(everyone, mine, group=group)
        self._opened = []  # (ptr, offset) mappings to close
        self.ptrs = [[0] * world for _ in range(2)]
        for i, b in enumerate(self.bufs):
            for r in range(world):
                if r == rank:
                    self.ptrs[i][r] = b.data_ptr()
                    continue
                handle, off = everyone[r][i]
                hb = (ct.c_char * L.IPC_HANDLE_BYTES).from_buffer_copy(handle)
                p = ct.c_void_p()
                L.check(L.lib.anima_ipc_open(hb, ct.c_uint64(off), ct.byref(p)), "anima_ipc_open")
                self.ptrs[i][r] = p.value
                self._opened.append((p.value, off))
        self._sync = torch.zeros(1, dtype=torch.float32, device=device)
        self.group = group

    def destinations(self, i: int, elem_offset: int) -> List[int]:
        """Bases of every rank's buffer i, moved by `elem_offset` elements (this rank's head
        columns), in rank order: the peer_out list of anima_attn_fwd_gather."""
        esz = self.bufs[i].element_size()
        return [p + elem_offset * esz for p in self.ptrs[i]]

    def barrier(self) -> None:
        """Orders the ranks on the current stream: when it completes on any rank, every
        rank's work queued before it (the attention kernel that stored into the buffers) has
        completed."""
        import torch.distributed as dist
        dist.all_reduce(self._sync, group=self.group)

    def close(self) -> None:
        for p, off in self._opened:
            L.lib.anima_ipc_close(ct.c_void_p(p), ct.c_uint64(off))
        self._opened = []
