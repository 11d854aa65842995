"""Pinned host slab and host-resident saved activations.

`PinnedSlab`: one page-locked host buffer, carved into 512-byte-aligned pieces for the
tensors of one training call and grown to the largest need seen (one registration
instead of one pinned allocation per saved tensor; pinning costs ~0.4 s/GiB, so the
slab is kept across calls and only grown).  `release()` drops the carve (not the pages).

`HostActivations`: autograd saved-tensor hooks that keep the first `gpu_budget` bytes
of saved activations on the GPU and copy the rest into the slab on a side stream
(device -> host), bringing them back on use in backward.  With per-layer (or block)
checkpointing the saved tensors are the layers' inputs, so GPU memory for activations
stays bounded by the budget plus one layer's working set.  Refuses to run without
checkpointing (every intermediate would go through host memory).

Reference parity (behaviour): `octopus/rl/pinned_slab.py:15-57`, host activations of
`octopus/rl/lm_head.py:156-199` and `octopus/rl/actor.py:116-150` (check_checkpointing).
"""
from __future__ import annotations

import torch

ALIGN = 512


class PinnedSlab:
    def __init__(self):
        self.buf: torch.Tensor | None = None
        self.off = 0

    def capacity(self) -> int:
        return 0 if self.buf is None else self.buf.numel()

    def reserve(self, nbytes: int):
        """Make sure the slab holds at least nbytes (grows; keeps pages across calls)."""
        if nbytes > self.capacity():
            pin = torch.cuda.is_available()
            self.buf = torch.empty(nbytes, dtype=torch.uint8, pin_memory=pin)
            self.off = 0

    def take(self, nbytes: int) -> torch.Tensor | None:
        """A byte view of the next free piece, or None when the slab is full."""
        a = (self.off + ALIGN - 1) // ALIGN * ALIGN
        if self.buf is None or a + nbytes > self.buf.numel():
            return None
        self.off = a + nbytes
        return self.buf[a: a + nbytes]

    def release(self):
        self.off = 0


class HostActivations:
    """saved_tensors_hooks context: saved activations past `gpu_budget` bytes live in host memory."""

    def __init__(self, gpu_budget: int, slab: PinnedSlab | None = None, min_bytes: int = 1 << 20):
        self.budget = gpu_budget
        self.slab = slab or PinnedSlab()
        self.min_bytes = min_bytes
        self.on_gpu = 0
        self.host_bytes = 0
        self.stream = torch.cuda.Stream() if torch.cuda.is_available() else None
        self._ctx = None

    def _pack(self, t: torch.Tensor):
        nb = t.numel() * t.element_size()
        if not t.is_cuda or nb < self.min_bytes or self.on_gpu + nb <= self.budget:
            self.on_gpu += nb if t.is_cuda else 0
            return ("dev", t)
        piece = self.slab.take(nb)
        host = piece.view(t.dtype)[: t.numel()].view(t.shape) if piece is not None else \
            torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        self.stream.wait_stream(torch.cuda.current_stream(t.device))
        with torch.cuda.stream(self.stream):
            host.copy_(t, non_blocking=True)
        t.record_stream(self.stream)
        ev = torch.cuda.Event()
        ev.record(self.stream)
        self.host_bytes += nb
        return ("host", host, t.device, ev)

    @staticmethod
    def _unpack(p):
        if p[0] == "dev":
            return p[1]
        _, host, dev, ev = p
        ev.synchronize()
        return host.to(dev, non_blocking=True)

    def __enter__(self):
        self.on_gpu = 0
        self.host_bytes = 0
        self.slab.release()
        self._ctx = torch.autograd.graph.saved_tensors_hooks(self._pack, self._unpack)
        self._ctx.__enter__()
        return self

    def __exit__(self, *exc):
        self._ctx.__exit__(*exc)
        self._ctx = None
        return False


def check_checkpointing(ckpt: bool, host: HostActivations | None):
    if host is not None and not ckpt:
        raise ValueError("host activations need layer checkpointing (every intermediate would cross PCIe)")
