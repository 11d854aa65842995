"""IPC peer buffers: one cudaMalloc'd buffer per rank of a process group, mapped into every
rank, so the fused kernels can load from and store to any rank's buffer over NVLink."""
from __future__ import annotations

import torch.distributed as dist

from .. import ops


class PeerBuffers:
    """One IPC-capable buffer per rank, mapped into every rank (device pointers)."""

    def __init__(self, nbytes: int, device: torch.device, group=None):
        C = ops.ext()
        self.local = C.symm_alloc(nbytes, device.index)
        handle = C.ipc_handle(self.local)
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        handles = [None] * world
        dist.all_gather_object(handles, handle, group=group)
        self.ptrs = []
        self._opened = []
        for r, h in enumerate(handles):
            if r == rank:
                self.ptrs.append(self.local.data_ptr())
            else:
                p = C.ipc_open(h, device.index)
                self.ptrs.append(p)
                self._opened.append(p)

    def close(self):
        C = ops.ext()
        for p in self._opened:
            C.ipc_close(p)
        self._opened = []
