"""Peer memory for the fused output gather across the GPUs of one node.

Every rank allocates the same gathered-output tensor.  ``PeerGather`` exports
this rank's copy through the library (``dash_peer_export``: CUDA IPC handle of
its allocation + offset), exchanges the handles over the process group and
imports every other rank's copy (``dash_peer_import``).  The prefill kernel
then stores each output row it finishes into the local copy and, over NVLink,
into every peer's copy at the same offset (``DashPrefillArgs.out_peers``), so
the gather runs inside the attention, tile by tile.  ``complete()`` orders a
one-word NCCL all-reduce after the kernels on the current stream: once it
finishes on a rank, every rank's kernel has ended (a grid completes only once
all of its writes, the posted peer stores included, are performed), so the
whole gathered tensor is in place.
"""
from __future__ import annotations

import ctypes as C
from typing import Dict, Optional

import torch
import torch.distributed as dist

from . import _lib as L


class PeerGather:
    def __init__(self, full: torch.Tensor, group: Optional[dist.ProcessGroup] = None):
        if not full.is_cuda:
            raise RuntimeError("PeerGather needs a CUDA tensor")
        self.full = full
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        lib = L.load()
        h = L.DashPeerHandle()
        if lib.dash_peer_export(C.c_void_p(full.data_ptr()), C.byref(h)) != L.DASH_OK:
            raise L.DashError(L.DASH_ERR_CUDA, L.last_error())
        mine = (bytes(h.handle), int(h.offset), int(h.alloc_bytes), full.numel() * full.element_size())
        every = [None] * self.world
        dist.all_gather_object(every, mine, group=group)
        self._bases = []
        self._imported = []
        for r, (hb, off, alloc, nbytes) in enumerate(every):
            if r == self.rank:
                continue
            if nbytes != mine[3]:
                raise RuntimeError(f"rank {r} gathered buffer has {nbytes} bytes, this rank {mine[3]}")
            ph = L.DashPeerHandle()
            ph.handle = (C.c_ubyte * 64)(*hb)
            ph.offset, ph.alloc_bytes = off, alloc
            p = C.c_void_p()
            if lib.dash_peer_import(C.byref(ph), C.byref(p)) != L.DASH_OK:
                raise L.DashError(L.DASH_ERR_CUDA, L.last_error())
            self._imported.append(p.value)
            self._bases.append(p.value)
        self._arrays: Dict[int, torch.Tensor] = {}
        self._flag = torch.zeros(1, dtype=torch.int32, device=full.device)

    @property
    def n_peers(self) -> int:
        return len(self._bases)

    def peers_for(self, view: torch.Tensor) -> torch.Tensor:
        """Device array (int64) of the peers' addresses of ``view``, a view into
        the local gathered tensor; cached per offset (build it before any CUDA
        graph capture)."""
        off = view.data_ptr() - self.full.data_ptr()
        if off < 0 or off >= self.full.numel() * self.full.element_size():
            raise ValueError("view does not lie inside the gathered tensor")
        arr = self._arrays.get(off)
        if arr is None:
            arr = torch.tensor([b + off for b in self._bases], dtype=torch.int64,
                               device=self.full.device)
            self._arrays[off] = arr
        return arr

    def complete(self) -> None:
        """Stream-ordered completion of the fused gather (see the module text)."""
        dist.all_reduce(self._flag, group=self.group)

    def close(self) -> None:
        """Unmap the peers' buffers once no rank can still be storing into them."""
        lib = L.load()
        torch.cuda.synchronize(self.full.device)
        dist.barrier(group=self.group)
        for p in self._imported:
            lib.dash_peer_close(C.c_void_p(p))
        self._imported, self._bases, self._arrays = [], [], {}
