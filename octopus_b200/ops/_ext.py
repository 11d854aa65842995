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


# Kernels launched by each entry point of the extension (for launch accounting).
KERNELS_PER_CALL = {
    "gemm_out": 1, "head_fwd": 2, "head_grad_logits": 1, "sample_head": 2, "rmsnorm_fwd": 1, "rmsnorm_bwd": 1,
    "rope": 1, "swiglu_fwd": 1, "swiglu_bwd": 1, "embed_fwd": 1, "embed_bwd": 1, "kv_write": 1,
    "sqnorm_accum": 1, "adamw": 1, "attn_fwd": 1, "attn_bwd": 3, "attn_decode": 2, "gemm_swiglu": 1, "gemm_rope": 1, "attn_decode_persistent": 2,
    "attn_decode_shared": 2, "recur_fwd": 1, "recur_bwd": 1, "conv_fwd": 1, "conv_bwd": 1,
    "rs_sum_sq": 1, "adamw_bcast": 1, "bcast_bf16": 1, "peer_barrier": 1, "peer_gather_bf16": 1, "peer_rs_acc": 1,
}
LAUNCHES = {"count": 0}


class _Counting:
    """Proxy of the extension module that counts kernel launches per call."""

    def __init__(self, mod):
        self._mod = mod
        self._cache = {}

    def __getattr__(self, name):
        fn = self._cache.get(name)
        if fn is None:
            target = getattr(self._mod, name)
            k = KERNELS_PER_CALL.get(name, 0)
            if not k or not callable(target):
                return target

            def fn(*a, _t=target, _k=k, **kw):
                LAUNCHES["count"] += _k
                return _t(*a, **kw)

            self._cache[name] = fn
        return fn


_PROXY = None


def ext():
    """Return the (launch-counting) extension module or raise a clear error."""
    global _PROXY
    mod = _load()
    if mod is None:
        raise RuntimeError(
            "octopus_b200._C (the sm_100a kernels) is not built or failed to load: "
            f"{_ERR!r}. Build it with `python setup.py build_ext --inplace`."
        )
    if _PROXY is None:
        _PROXY = _Counting(mod)
    return _PROXY


def launches() -> int:
    """Kernels of this extension launched from Python so far (graph replays excluded)."""
    return LAUNCHES["count"]


def add_launches(n: int) -> None:
    """Account kernels launched by CUDA-graph replays of captured extension calls."""
    LAUNCHES["count"] += int(n)


def available() -> bool:
    return _load() is not None


ERR_NAMES = {1: "pipeline barrier wait timed out", 2: "peer flag wait timed out", 3: "bounds check failed",
             4: "TMEM allocation failed"}


class KernelError(RuntimeError):
    """A kernel recorded an error in the device status word (the context is still usable)."""

    def __init__(self, code: int, where: int, index: int):
        self.code, self.where, self.index = code, where, index
        extra = f", index {index}" if code == 3 else ""
        super().__init__(f"octopus_b200 kernel error {code} ({ERR_NAMES.get(code, '?')}) at site {where}{extra}")


def read_status(device: int = 0) -> tuple[int, int, int]:
    """(code, site, rejected index) of the device status word, without clearing it (syncs)."""
    code, where, _budget, index = (int(x) for x in ext().status_tensor(device).cpu().tolist())
    return code, where, index


def check_status(device: int = 0, reset: bool = True) -> None:
    """Raise KernelError if a kernel on `device` recorded a timeout or bounds error (syncs)."""
    code, where, index = read_status(device)
    if reset and code:
        st = ext().status_tensor(device)
        st[0:2].zero_()
        st[3:4].zero_()
    if code:
        raise KernelError(code, where, index)


def set_wait_budget(device: int, microseconds: int) -> int:
    """Set the time limit of every primary device-side wait on `device` (mbarrier phases,
    peer flags, staging counters); 0 restores the compiled default (2 s).  Returns the
    previous value.  Stream-ordered: it applies to kernels launched afterwards on the
    current stream."""
    st = ext().status_tensor(device)
    prev = int(st[2].item())
    st[2:3].fill_(int(microseconds))
    return prev


class wait_budget:
    """Context: a runtime wait budget (microseconds) for kernels launched inside."""

    def __init__(self, device: int, microseconds: int):
        self.device, self.us = device, microseconds

    def __enter__(self):
        self.prev = set_wait_budget(self.device, self.us)
        return self

    def __exit__(self, *exc):
        set_wait_budget(self.device, self.prev)
        return False


class pdl_launches:
    """Context: GEMMs launched inside are programmatic dependents of the preceding kernel
    (their prologue and weight L2 prefetch overlap its tail).  Used for the engine's
    decode graphs; OCTO_PDL=0 disables it."""

    def __enter__(self):
        import os

        self.on = os.environ.get("OCTO_PDL", "1") != "0" and available()
        if self.on:
            ext().set_pdl(True)
        return self

    def __exit__(self, *exc):
        if self.on:
            ext().set_pdl(False)
        return False
