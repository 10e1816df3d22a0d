"""Builds and loads the sm_100a kernel library (``ops/csrc``) in-tree.

``all_kernels.cu`` (every kernel source, one translation unit) is compiled with
``nvcc -gencode arch=compute_100a,code=sm_100a`` and linked with the torch bindings into
``maloq_b200/ops/build/maloq_b200_C.so``.  Building needs no GPU.  On a machine with a GPU
the ops raise if the library cannot be built or loaded - there is no fallback.
"""

from __future__ import annotations

import os

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "build")
NAME = "maloq_b200_C"
CUDA_FLAGS = ["-gencode=arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr"]
_mod = None


def sources():
    return [os.path.join(CSRC, "all_kernels.cu"), os.path.join(CSRC, "bindings.cpp")]


def load(verbose: bool = False):
    global _mod
    if _mod is not None:
        return _mod
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    os.makedirs(BUILD, exist_ok=True)
    from torch.utils.cpp_extension import load as _load

    _mod = _load(name=NAME, sources=sources(), build_directory=BUILD, extra_cuda_cflags=CUDA_FLAGS,
                 extra_cflags=["-O3", "-std=c++17"], extra_include_paths=[CSRC], verbose=verbose)
    return _mod
