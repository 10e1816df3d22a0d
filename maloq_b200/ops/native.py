"""CUDA implementations (sm_100a kernels) behind the op layer; filled in by ops/cuda_*.py."""
from __future__ import annotations

_IMPL = {}


def register(name):
    def deco(fn):
        _IMPL[name] = fn
        return fn
    return deco


def _get(name):
    fn = _IMPL.get(name)
    if fn is None:
        from . import kernels  # noqa: F401  (registers the kernel-backed ops)
        fn = _IMPL.get(name)
    if fn is None:
        raise RuntimeError(f"maloq_b200: no CUDA kernel registered for op {name!r}")
    return fn


def __getattr__(name):
    if name.startswith("_"):
        raise AttributeError(name)
    return _get(name)
