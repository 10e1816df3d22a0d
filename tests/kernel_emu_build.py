"""Build the emulated (CPU) versions of kernel source files for tests: the ops/csrc sources are
rewritten textually - launch syntax to the emulator's launch operators, shared-memory
declarations to block-shared storage, tests/csrc/host_emu.cuh in place of common.cuh - and
compiled with the host compiler together with a file of extern "C" entry points.  The
production sources are not modified."""

from __future__ import annotations

import ctypes
import os
import re
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "..", "maloq_b200", "ops", "csrc")
CUDA_INC = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")


def rewrite(text):
    text = text.replace('#include "common.cuh"', '#include "host_emu.cuh"')
    # kernel<...><<<grid, block, smem, stream>>>(args)  ->  kernel<...> ^ Cfg(...) | args(...)
    text = text.replace("<<<", " ^ ::emu::Cfg(").replace(">>>(", ") | ::emu::args(")
    text = re.sub(r"extern __shared__\s+(?:__align__\(\d+\)\s+)?((?:unsigned\s+)?[\w:]+)\s+(\w+)\[\];",
                  r"\1* \2 = reinterpret_cast<\1*>(::emu::dyn_smem());", text)
    text = text.replace("__shared__ ", "static ")
    return text


def build(name, out_dir, defines=()):
    """Compile tests/csrc/<name>_emu.cpp with the rewritten ops/csrc/<name>.cu (extra ``-D``
    ``defines``); returns the CDLL."""
    cxx = shutil.which("g++")
    if cxx is None or not os.path.isfile(os.path.join(CUDA_INC, "cuda_bf16.h")):
        return None
    with open(os.path.join(CSRC, f"{name}.cu")) as fh:
        src = rewrite(fh.read())
    with open(os.path.join(out_dir, f"{name}_emu_src.inc"), "w") as fh:
        fh.write(src)
    tag = "".join("_" + d.split("=")[0].lower() for d in defines)
    so = os.path.join(out_dir, f"{name}_emu{tag}.so")
    cmd = [cxx, "-O1", "-std=c++20", "-shared", "-fPIC", "-w", "-pthread", "-DMALOQ_HOST_EMULATION=1", *("-D" + d for d in defines),
           "-I", out_dir, "-I", os.path.join(HERE, "csrc"), "-I", CSRC, "-I", CUDA_INC,
           os.path.join(HERE, "csrc", f"{name}_emu.cpp"), "-o", so]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(r.stderr[-6000:])
    lib = ctypes.CDLL(so)
    return lib
