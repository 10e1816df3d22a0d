"""Radius graph built on the device (cell list, CUDA kernels in ``ops/csrc/graph.cu``).

Same conventions and edge order as :func:`maloq_b200.data.graph.radius_graph` (pair cutoff,
``vec = pos[src] - pos[dst]`` with the minimum image in a periodic orthorhombic cell, no self
edges, sorted by (dst, src)); ``targets`` restricts the destinations to a subset of atoms (one
rank's owned atoms in a partitioned run), and ``dst`` then indexes ``targets``.  Used for
structures too large for the host builder (the 10^6-atom inference config builds ~10^8 edges).
"""

from __future__ import annotations

import numpy as np
import torch


def grid_for(pos, cutoff, cell=None):
    """(lo, ext, ncell, periodic) of the cell list: cells of edge >= cutoff over the periodic
    cell, or over the bounding box of open structures."""
    pos = np.asarray(pos, dtype=np.float64)
    if cell is not None:
        cell = np.asarray(cell, dtype=np.float64)
        if np.any(cell < 2 * cutoff):
            raise ValueError("periodic cell must be at least twice the cutoff (single image)")
        lo, ext, periodic = np.zeros(3), cell, [1, 1, 1]
    else:
        lo = pos.min(axis=0)
        ext = pos.max(axis=0) - lo + 1e-9
        periodic = [0, 0, 0]
    ncell = np.maximum((ext / cutoff).astype(np.int64), 1)
    return lo, ext, ncell, periodic


def radius_graph_device(pos, cutoff, cell=None, targets=None, device="cuda"):
    """Return (src, dst, vec, dst_ptr) as device tensors (int64, int64, float64 [E, 3], int64
    [n_targets + 1])."""
    from ..ops.kernels import lib
    from ..ops.native import count_launches

    L = lib()
    pos_np = np.asarray(pos, dtype=np.float64)
    n = len(pos_np)
    dev = torch.device(device)
    lo, ext, ncell, periodic = grid_for(pos_np, cutoff, cell)
    grid = [float(v) for v in lo] + [float(v) for v in ext] + [float(cutoff)]
    nc = [int(v) for v in ncell]
    pos_t = torch.as_tensor(pos_np, device=dev).contiguous()
    cell_id = torch.empty(n, dtype=torch.long, device=dev)
    L.radius_graph_cells(pos_t, grid, nc, periodic, cell_id)
    order = torch.argsort(cell_id, stable=True)
    n_cells = nc[0] * nc[1] * nc[2]
    cell_start = torch.zeros(n_cells + 1, dtype=torch.long, device=dev)
    cell_start[1:] = torch.cumsum(torch.bincount(cell_id, minlength=n_cells), 0)
    tg = torch.arange(n, device=dev) if targets is None else torch.as_tensor(targets, dtype=torch.long, device=dev)
    tg = tg.contiguous()
    counts = torch.empty(tg.numel(), dtype=torch.long, device=dev)
    L.radius_graph_pass(pos_t, grid, nc, periodic, tg, order, cell_start, counts, None, None, None)
    ptr = torch.zeros(tg.numel() + 1, dtype=torch.long, device=dev)
    ptr[1:] = torch.cumsum(counts, 0)
    E = int(ptr[-1])
    src = torch.empty(E, dtype=torch.long, device=dev)
    vec = torch.empty(E, 3, dtype=torch.float64, device=dev)
    L.radius_graph_pass(pos_t, grid, nc, periodic, tg, order, cell_start, None, ptr[:-1].contiguous(), src, vec)
    count_launches(3)
    dst = torch.repeat_interleave(torch.arange(tg.numel(), device=dev), counts)
    o = torch.argsort(dst * n + src)  # (dst, src) order within the dst-major layout
    return src[o], dst, vec[o], ptr
