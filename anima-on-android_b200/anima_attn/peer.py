"""Buffers shared by the ranks of one node over NVLink (CUDA IPC), for collectives folded
into the kernels that produce their data.

PeerBuffers allocates named tensors on every rank and maps every rank's copy into every
rank (peer access over NVLink).  Kernels of this library then store straight into other
ranks' buffers -- the attention epilogue's all-gather of head outputs
(anima_attn_fwd_gather), the projection GEMM's and the attention's all-to-alls
(anima_qkv_projection_scatter, anima_attn_fwd_scatter_rows) -- and a one-element all-reduce
on the stream orders the ranks before anyone reads what was stored (barrier()).

A rank writes a buffer of another rank only between two barriers that the reader also
passes, so a buffer that is read after barrier k is written again only after barrier k+1;
callers alternate two sets of buffers between consecutive collectives for this.
"""
from __future__ import annotations

import ctypes as ct
from typing import Dict, List, Tuple

import torch

from . import _lib as L


class PeerBuffers:
    """Named tensors {name: (shape, dtype)} on this rank's device, mapped into every rank.

    ``ptr(name, r)`` is the device address of rank r's tensor `name` in this process.  Every
    rank of ``group`` constructs it with the same specs in the same order; call ``close()``
    (every rank) before the process group is destroyed."""

    def __init__(self, specs: Dict[str, Tuple[tuple, torch.dtype]], device, group, rank: int,
                 world: int):
        import torch.distributed as dist
        self.rank, self.world, self.group = rank, world, group
        self.names = list(specs)
        self.local: Dict[str, torch.Tensor] = {
            n: torch.zeros(shape, dtype=dt, device=device) for n, (shape, dt) in specs.items()}
        mine = []
        for n in self.names:
            h = (ct.c_char * L.IPC_HANDLE_BYTES)()
            off = ct.c_uint64(0)
            L.check(L.lib.anima_ipc_export(ct.c_void_p(self.local[n].data_ptr()), h, ct.byref(off)),
                    "anima_ipc_export")
            mine.append((bytes(h), int(off.value)))
        everyone: List = [None] * world
        dist.all_gather_object(everyone, mine, group=group)
        self._opened = []  # (ptr, offset) mappings to close
        self._ptrs: Dict[str, List[int]] = {}
        for i, n in enumerate(self.names):
            row = []
            for r in range(world):
                if r == rank:
                    row.append(self.local[n].data_ptr())
                    continue
                handle, off = everyone[r][i]
                hb = (ct.c_char * L.IPC_HANDLE_BYTES).from_buffer_copy(handle)
                p = ct.c_void_p()
                L.check(L.lib.anima_ipc_open(hb, ct.c_uint64(off), ct.byref(p)), "anima_ipc_open")
                row.append(p.value)
                self._opened.append((p.value, off))
            self._ptrs[n] = row
        self._sync = torch.zeros(1, dtype=torch.float32, device=device)

    def ptr(self, name: str, r: int) -> int:
        return self._ptrs[name][r]

    def ptrs(self, name: str, elem_offset: int = 0) -> List[int]:
        """Every rank's tensor `name`, moved by `elem_offset` elements, in rank order."""
        esz = self.local[name].element_size()
        return [p + elem_offset * esz for p in self._ptrs[name]]

    def barrier(self) -> None:
        """Orders the ranks on the current stream: when it completes on any rank, every
        rank's work queued before it (the kernels that stored into the buffers) has
        completed."""
        import torch.distributed as dist
        dist.all_reduce(self._sync, group=self.group)

    def close(self) -> None:
        for p, off in self._opened:
            L.lib.anima_ipc_close(ct.c_void_p(p), ct.c_uint64(off))
        self._opened = []


class GatherBuffers(PeerBuffers):
    """Two [B, S, H, D] buffers (``bufs[0]``, ``bufs[1]``) for the head-parallel step's
    all-gather of attention outputs, which alternate between consecutive attentions."""

    def __init__(self, shape, dtype: torch.dtype, device, group, rank: int, world: int):
        super().__init__({"g0": (tuple(shape), dtype), "g1": (tuple(shape), dtype)}, device,
                         group, rank, world)
        self.bufs = [self.local["g0"], self.local["g1"]]

    def destinations(self, i: int, elem_offset: int) -> List[int]:
        """Bases of every rank's buffer i, moved by `elem_offset` elements (this rank's head
        columns), in rank order: the peer_out list of anima_attn_fwd_gather."""
        return self.ptrs(f"g{i}", elem_offset)
