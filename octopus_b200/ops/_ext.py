"""Loader of the in-tree CUDA extension ``octopus_b200._C``.

CUDA tensors always go through the extension: if it is missing or fails to load, a
CUDA call raises instead of silently falling back to PyTorch.  CPU tensors use the
plain-PyTorch reference implementations in :mod:`octopus_b200.ops.reference`, which
the CPU test-suite runs.
"""
from __future__ import annotations

import importlib

_C = None
_ERR: Exception | None = None


def _load():
    global _C, _ERR
    if _C is not None or _ERR is not None:
        return _C
    try:
        _C = importlib.import_module("octopus_b200._C")
    except Exception as e:  # pragma: no cover - depends on the build
        _ERR = e
    return _C


def ext():
    """Return the extension module or raise a clear error."""
    mod = _load()
    if mod is None:
        raise RuntimeError(
            "octopus_b200._C (the sm_100a kernels) is not built or failed to load: "
            f"{_ERR!r}. Build it with `python setup.py build_ext --inplace`."
        )
    return mod


def available() -> bool:
    return _load() is not None


def check_status(device: int = 0, reset: bool = True) -> None:
    """Raise if a kernel on `device` recorded a timeout or bounds error (syncs)."""
    st = ext().status_tensor(device)
    code, where = (int(x) for x in st.cpu().tolist())
    if reset and code:
        st.zero_()
    if code:
        names = {1: "pipeline barrier wait timed out", 2: "peer flag wait timed out",
                 3: "bounds check failed", 4: "TMEM allocation failed"}
        raise RuntimeError(f"octopus_b200 kernel error {code} ({names.get(code, '?')}) at site {where}")
