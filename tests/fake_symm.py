"""Symmetric memory emulated in host shared memory, for multi-process CPU tests.

The NVLink paths (peer halo, fused gradient all-reduce) allocate buffers with
``torch.distributed._symmetric_memory`` and hand the kernels tables of every rank's buffer
address.  Here each rank's buffer is a file-backed shared-memory tensor; ``rendezvous`` maps
every rank's file into this process, so the address table holds addresses valid in this process
- as device peer pointers are in the real one - and the CPU stand-in kernels
(``tests/cpu_extension.py``) read and write peers' memory through them, spin on signal pads
written by other processes, and time out like the bounded device waits.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np
import torch
import torch.distributed as dist

PAD_WORDS = 1024  # uint32 signal slots per rank


class _Handle:
    def __init__(self, bufs, pads):
        self._bufs, self._pads = bufs, pads  # keep the mappings alive
        self.buffer_ptrs = [b.data_ptr() for b in bufs]
        self.signal_pad_ptrs = [p.data_ptr() for p in pads]
        self.multicast_ptr = 0

    def barrier(self, *args, **kwargs):
        dist.barrier()


class FakeSymmetricMemory:
    """Stand-in for ``torch.distributed._symmetric_memory`` (``empty`` / ``rendezvous``)."""

    def __init__(self, folder):
        self.folder = folder
        self.seq = 0
        self._files = {}

    def empty(self, n, dtype=torch.float32, device=None):
        rank = dist.get_rank()
        path = os.path.join(self.folder, f"r{rank}_{self.seq}.bin")
        self.seq += 1
        nbytes = int(n) * torch.empty(0, dtype=dtype).element_size()
        with open(path, "wb") as fh:
            fh.truncate(max(nbytes, 16))
        t = torch.from_file(path, shared=True, size=int(n), dtype=dtype)
        self._files[t.data_ptr()] = (path, int(n), dtype)
        return t

    def rendezvous(self, buf, group_name=None):
        rank, world = dist.get_rank(), dist.get_world_size()
        path, n, dtype = self._files[buf.data_ptr()]
        pad_path = path + ".pad"
        with open(pad_path, "wb") as fh:
            fh.truncate(4 * PAD_WORDS)
        info = [None] * world
        dist.all_gather_object(info, (path, pad_path, n, str(dtype)))
        bufs, pads = [], []
        for r, (p, pp, nn, _) in enumerate(info):
            bufs.append(buf if r == rank else torch.from_file(p, shared=True, size=nn, dtype=dtype))
            pads.append(torch.from_file(pp, shared=True, size=PAD_WORDS, dtype=torch.int32))
        dist.barrier()
        return _Handle(bufs, pads)


def install(folder):
    """Make ``torch.distributed._symmetric_memory`` resolve to the emulation in this process."""
    import sys

    os.makedirs(folder, exist_ok=True)
    fake = FakeSymmetricMemory(folder)
    sys.modules["torch.distributed._symmetric_memory"] = fake
    torch.distributed._symmetric_memory = fake
    return fake


# ------------------------------------------------------------------ raw-address views
def floats_at(addr, n):
    """A float32 tensor viewing n values at host address ``addr`` (shared memory)."""
    return torch.from_numpy(np.ctypeslib.as_array((ctypes.c_float * int(n)).from_address(int(addr))))


def int32_at(addr, n):
    return np.ctypeslib.as_array((ctypes.c_int32 * int(n)).from_address(int(addr)))


def table(addr, n):
    """The n int64 addresses of a pointer table stored at ``addr``."""
    return list(np.ctypeslib.as_array((ctypes.c_int64 * int(n)).from_address(int(addr))))
