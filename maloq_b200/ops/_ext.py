"""Builds and loads the sm_100a kernel library (``ops/csrc``) in-tree.

``all_kernels.cu`` (every kernel source, one translation unit) is compiled with
``nvcc -gencode arch=compute_100a,code=sm_100a`` and linked with the torch bindings into
``maloq_b200/ops/build/maloq_b200_C.so``.  Building needs no GPU.  On a machine with a GPU
the ops raise if the library cannot be built or loaded - there is no fallback.

``MALOQ_BOUNDS_CHECK=1`` loads a second build (``build_checked/maloq_b200_C_checked.so``,
compiled with ``-DMALOQ_BOUNDS_CHECK``) whose kernels check data-dependent indices (gather
sources/destinations, segment offsets, pair types, block offsets) and record error code 5
instead of accessing out of range.
"""

from __future__ import annotations

import os

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "build")
NAME = "maloq_b200_C"
CUDA_FLAGS = ["-gencode=arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr"]
_mods = {}


def checked_requested() -> bool:
    return os.environ.get("MALOQ_BOUNDS_CHECK", "0") not in ("", "0")


def sources():
    return [os.path.join(CSRC, "all_kernels.cu"), os.path.join(CSRC, "bindings.cpp")]


def load(verbose: bool = False, checked: bool | None = None):
    """The kernel library (built on first use); ``checked`` selects the bounds-checked build
    (default: the ``MALOQ_BOUNDS_CHECK`` environment variable)."""
    checked = checked_requested() if checked is None else checked
    if checked in _mods:
        return _mods[checked]
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    build = BUILD + ("_checked" if checked else "")
    os.makedirs(build, exist_ok=True)
    from torch.utils.cpp_extension import load as _load

    flags = CUDA_FLAGS + (["-DMALOQ_BOUNDS_CHECK"] if checked else [])
    _mods[checked] = _load(name=NAME + ("_checked" if checked else ""), sources=sources(), build_directory=build,
                           extra_cuda_cflags=flags, extra_cflags=["-O3", "-std=c++17"], extra_include_paths=[CSRC],
                           verbose=verbose)
    return _mods[checked]
