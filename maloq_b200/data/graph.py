"""Radius graphs on the host (cell list), periodic (orthorhombic, minimum image) or open.

Replaces the reference's ASE ``NeighborList`` (``fock_targets_batched.py:189-229``).
Conventions kept from the reference:

* ``cutoff`` is the pair distance (the reference's per-atom ``rcut_orbitals`` radius is
  converted by the caller: pair cutoff = 2 * rcut_orbitals);
* edge ``e`` carries ``edge_attr[e] = [d, dx, dy, dz]`` with ``(dx, dy, dz) = pos[src] -
  pos[dst]`` (minimum image), and messages flow src -> dst;
* no self edges; both directions present.

Edges are returned sorted by ``dst`` (then ``src``), the order the segmented-reduction
kernels need.  Structures too large for this builder use the device builder
(:mod:`maloq_b200.data.graph_gpu`), which gives the same edges in the same order.
"""

from __future__ import annotations

import numpy as np


def radius_graph(pos, cutoff, cell=None, chunk=65536):
    """Return (src, dst, vec) with vec = pos[src] - pos[dst] (minimum image if ``cell``)."""
    pos = np.ascontiguousarray(pos, dtype=np.float64)
    n = len(pos)
    if n == 0:
        return np.zeros(0, np.int64), np.zeros(0, np.int64), np.zeros((0, 3))
    if cell is not None:
        cell = np.asarray(cell, dtype=np.float64)
        if np.any(cell < 2 * cutoff):
            raise ValueError("periodic cell must be at least twice the cutoff (single image)")
        lo = np.zeros(3)
        ext = cell
        p = np.mod(pos, cell)
    else:
        lo = pos.min(axis=0)
        ext = pos.max(axis=0) - lo + 1e-9
        p = pos - lo
    ncell = np.maximum((ext / cutoff).astype(np.int64), 1)
    if cell is not None:
        ncell = np.maximum(ncell, 1)
    cidx = np.minimum((p / (ext / ncell)).astype(np.int64), ncell - 1)
    flat = (cidx[:, 0] * ncell[1] + cidx[:, 1]) * ncell[2] + cidx[:, 2]
    order = np.argsort(flat, kind="stable")
    counts = np.bincount(flat, minlength=int(np.prod(ncell)))
    starts = np.concatenate([[0], np.cumsum(counts)])
    offs = np.array([(a, b, c) for a in (-1, 0, 1) for b in (-1, 0, 1) for c in (-1, 0, 1)])
    if cell is None:
        # dedupe offsets that wrap onto the same cell along a dimension of size < 3
        pass
    srcs, dsts, vecs = [], [], []
    c2 = cutoff * cutoff
    for s in range(0, n, chunk):
        i = np.arange(s, min(n, s + chunk))
        ci = cidx[i]
        seen = set()
        for o in offs:
            nb = ci + o
            if cell is not None:
                nb = np.mod(nb, ncell)
                # skip duplicate neighbour cells when ncell < 3 along an axis
                key = tuple(np.mod(o, ncell))
                if key in seen:
                    continue
                seen.add(key)
                valid = np.ones(len(i), dtype=bool)
            else:
                valid = np.all((nb >= 0) & (nb < ncell), axis=1)
            ii = i[valid]
            nbf = ((nb[valid, 0] * ncell[1] + nb[valid, 1]) * ncell[2] + nb[valid, 2])
            cnt = counts[nbf]
            if cnt.sum() == 0:
                continue
            rep_i = np.repeat(ii, cnt)
            base = np.repeat(starts[nbf], cnt)
            within = np.arange(cnt.sum()) - np.repeat(np.cumsum(cnt) - cnt, cnt)
            j = order[base + within]
            d = pos[j] - pos[rep_i]  # vec for edge j -> i : pos[src] - pos[dst]
            if cell is not None:
                d -= cell * np.round(d / cell)
            r2 = (d * d).sum(axis=1)
            keep = (r2 < c2) & (j != rep_i)
            srcs.append(j[keep])
            dsts.append(rep_i[keep])
            vecs.append(d[keep])
    src = np.concatenate(srcs) if srcs else np.zeros(0, np.int64)
    dst = np.concatenate(dsts) if dsts else np.zeros(0, np.int64)
    vec = np.concatenate(vecs) if vecs else np.zeros((0, 3))
    o = np.lexsort((src, dst))
    return src[o].astype(np.int64), dst[o].astype(np.int64), vec[o]


def edge_attr_from_vec(vec):
    vec = np.asarray(vec, dtype=np.float64)
    d = np.linalg.norm(vec, axis=1, keepdims=True)
    return np.concatenate([d, vec], axis=1)


def dst_pointer(dst, num_nodes):
    """CSR offsets of dst-sorted edges: edges of node v are dst_ptr[v]:dst_ptr[v+1]."""
    counts = np.bincount(dst, minlength=num_nodes)
    return np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
