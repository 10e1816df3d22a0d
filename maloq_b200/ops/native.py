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
