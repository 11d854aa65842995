"""Host<->device transfer accounting and pinned staging.

Every host->device copy of step inputs made by the engine and the trainer goes through
:func:`h2d` (numpy -> pinned host tensor -> async device copy) and every device->host
result read through :func:`d2h`, so a benchmark can report the bytes that crossed PCIe
per step.
"""
from __future__ import annotations

import threading

import numpy as np
import torch

_lock = threading.Lock()
_counts = {"h2d": 0, "d2h": 0}


def reset():
    with _lock:
        _counts["h2d"] = 0
        _counts["d2h"] = 0


def snapshot() -> dict:
    with _lock:
        return dict(_counts)


def h2d(a, device, dtype=None) -> torch.Tensor:
    """Copy a numpy array / CPU tensor to `device` via pinned memory (counted)."""
    t = torch.from_numpy(np.ascontiguousarray(a)) if isinstance(a, np.ndarray) else a
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    dev = torch.device(device)
    if dev.type != "cuda":
        return t.to(dev)
    with _lock:
        _counts["h2d"] += t.numel() * t.element_size()
    return t.pin_memory().to(dev, non_blocking=True)


def d2h(t: torch.Tensor) -> torch.Tensor:
    if t.is_cuda:
        with _lock:
            _counts["d2h"] += t.numel() * t.element_size()
    return t.cpu()
