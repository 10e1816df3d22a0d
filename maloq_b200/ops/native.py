"""CUDA implementations (sm_100a kernels) behind the op layer (registered by ``ops/kernels.py``).

``MALOQ_NVTX=1`` puts every kernel-backed op call in an NVTX range ``maloq::<op>``."""
from __future__ import annotations

import os

_IMPL = {}


def register(name):
    def deco(fn):
        _IMPL[name] = fn
        return fn
    return deco


def _nvtx_wrap(name, fn):
    """``fn`` inside an NVTX range ``maloq::<op>`` (visible in Nsight timelines)."""
    import functools

    import torch

    @functools.wraps(fn)
    def wrapped(*args, **kwargs):
        torch.cuda.nvtx.range_push(f"maloq::{name}")
        try:
            return fn(*args, **kwargs)
        finally:
            torch.cuda.nvtx.range_pop()

    return wrapped


def _get(name):
    fn = _IMPL.get(name)
    if fn is None:
        from . import kernels  # noqa: F401  (registers the kernel-backed ops)
        fn = _IMPL.get(name)
    if fn is None:
        raise RuntimeError(f"maloq_b200: no CUDA kernel registered for op {name!r}")
    if os.environ.get("MALOQ_NVTX", "0") not in ("", "0"):
        fn = _nvtx_wrap(name, fn)
    return fn


def __getattr__(name):  # noqa: D401 - module-level op lookup
    if name.startswith("_"):
        raise AttributeError(name)
    return _get(name)


_LAUNCHES = [0]


def count_launches(n: int = 1) -> None:
    """Called by every kernel wrapper with the number of kernels it launched."""
    _LAUNCHES[0] += n


def launch_count() -> int:
    return _LAUNCHES[0]
