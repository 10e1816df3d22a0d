"""Graph partitioners and domain decomposition for graph-partitioned runs.

Ownership rule (reference ``fock_utils/domain_decomp.py:49-55``): a rank owns a set of
nodes and every edge whose destination it owns, so message aggregation is local and only
source-node ("halo") features cross ranks.

Partitioners (reference ``fock_utils/reorder.py:1209-1358``, ``domain_decomp.py:97-225``),
all returning ``part[node] -> rank``:

* ``linear-atomwise`` - contiguous index ranges with equal node counts;
* ``linear-edgewise`` - contiguous ranges with equal incoming-edge counts;
* ``slab`` - sort along the longest extent of the structure, cut into slabs with equal edge
  counts (spatial; periodic slabs touch their neighbours only);
* ``rcb`` - recursive coordinate bisection along the longest extent, edge-balanced (the
  reference's low_nn / longest_dim family);
* ``greedy`` - breadth-first region growing to equal edge counts (a dependency-free stand-in
  for METIS, which is not installed);
* ``worst-case`` - round-robin assignment (maximal cut), for stress tests.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


def _balanced_cuts(weights, parts):
    """Cut positions splitting a weight sequence into `parts` ranges of equal total weight."""
    c = np.cumsum(weights, dtype=np.float64)
    total = c[-1] if len(c) else 0.0
    targets = total * np.arange(1, parts) / parts
    return np.searchsorted(c, targets, side="left") + 1


def partition_linear_atomwise(n, world, **_):
    return np.minimum(np.arange(n) * world // max(n, 1), world - 1).astype(np.int64)


def partition_linear_edgewise(n, world, dst=None, **_):
    deg = np.bincount(dst, minlength=n) + 1
    cuts = _balanced_cuts(deg, world)
    part = np.zeros(n, dtype=np.int64)
    for r, c in enumerate(cuts):
        part[c:] = r + 1
    return part


def partition_slab(n, world, pos=None, dst=None, cell=None, **_):
    ext = np.ptp(pos, axis=0) if cell is None else np.asarray(cell)
    ax = int(np.argmax(ext))
    order = np.argsort(pos[:, ax], kind="stable")
    # balance in-degree + 1 per rank (equal atom counts when no edge list exists yet)
    deg = np.bincount(dst, minlength=n) + 1 if dst is not None else np.ones(n, dtype=np.int64)
    cuts = _balanced_cuts(deg[order], world)
    part = np.zeros(n, dtype=np.int64)
    bounds = [0] + list(cuts) + [n]
    for r in range(world):
        part[order[bounds[r]:bounds[r + 1]]] = r
    return part


def partition_rcb(n, world, pos=None, dst=None, **_):
    deg = np.bincount(dst, minlength=n) + 1
    part = np.zeros(n, dtype=np.int64)

    def rec(idx, lo, k):
        if k == 1:
            part[idx] = lo
            return
        ax = int(np.argmax(np.ptp(pos[idx], axis=0)))
        order = idx[np.argsort(pos[idx, ax], kind="stable")]
        k1 = k // 2
        c = np.cumsum(deg[order])
        cut = int(np.searchsorted(c, c[-1] * k1 / k)) + 1
        rec(order[:cut], lo, k1)
        rec(order[cut:], lo + k1, k - k1)

    rec(np.arange(n), 0, world)
    return part


def partition_greedy(n, world, src=None, dst=None, **_):
    deg = np.bincount(dst, minlength=n) + 1
    target = deg.sum() / world
    nbr_ptr = np.concatenate([[0], np.cumsum(np.bincount(dst, minlength=n))])
    nbrs = src[np.argsort(dst, kind="stable")]
    part = np.full(n, -1, dtype=np.int64)
    r, load = 0, 0.0
    from collections import deque

    for seed in range(n):
        if part[seed] >= 0:
            continue
        q = deque([seed])
        while q:
            v = q.popleft()
            if part[v] >= 0:
                continue
            part[v] = r
            load += deg[v]
            if load >= target and r < world - 1:
                r, load = r + 1, 0.0
                q.clear()
                break
            q.extend(u for u in nbrs[nbr_ptr[v]:nbr_ptr[v + 1]] if part[u] < 0)
    return part


def partition_worst_case(n, world, **_):
    return (np.arange(n) % world).astype(np.int64)


PARTITIONERS = {
    "linear-atomwise": partition_linear_atomwise, "linear-edgewise": partition_linear_edgewise,
    "slab": partition_slab, "rcb": partition_rcb, "low_nn": partition_rcb, "longest_dim": partition_rcb,
    "greedy": partition_greedy, "metis": partition_greedy, "worst-case": partition_worst_case,
}


def partition(name, n, world, **kw):
    if name not in PARTITIONERS:
        raise ValueError(f"unknown partition_type {name!r}; choose from {sorted(PARTITIONERS)}")
    part = PARTITIONERS[name](n, world, **kw)
    if world > 1 and len(np.unique(part)) < min(world, n):
        raise ValueError(f"partitioner {name!r} left a rank without nodes")
    return part


@dataclass
class Domain:
    """What one rank holds of a partitioned graph.

    ``owned``: global ids of owned nodes (sorted); ``edges``: global ids of local edges
    (dst owned), sorted by (local dst, src); ``halo``: global ids of non-owned source nodes;
    ``halo_owner`` / ``halo_row``: owning rank and that rank's local row of each halo node;
    ``src_local``: source of each local edge in the extended space [owned | halo];
    ``dst_local``: destination (owned local row); ``send[p]``: my local rows that rank p
    needs, in the order of p's halo list for me.
    """

    rank: int
    world: int
    owned: np.ndarray
    edges: np.ndarray
    halo: np.ndarray
    halo_owner: np.ndarray
    halo_row: np.ndarray
    src_local: np.ndarray
    dst_local: np.ndarray
    recv_counts: list = field(default_factory=list)
    send: list = field(default_factory=list)

    @property
    def n_own(self):
        return len(self.owned)

    @property
    def n_ext(self):
        return len(self.owned) + len(self.halo)


def decompose(part, src, dst, world):
    """Per-rank :class:`Domain` for a global graph with edges src -> dst (dst-sorted or not)."""
    n = len(part)
    local_row = np.zeros(n, dtype=np.int64)
    owned = [np.flatnonzero(part == r) for r in range(world)]
    for r in range(world):
        local_row[owned[r]] = np.arange(len(owned[r]))
    doms = []
    for r in range(world):
        eids = np.flatnonzero(part[dst] == r)
        s, d = src[eids], dst[eids]
        dl = local_row[d]
        order = np.lexsort((s, dl))
        eids, s, dl = eids[order], s[order], dl[order]
        remote = part[s] != r
        halo = np.unique(s[remote])
        # order halo by (owner, owner row) so each peer's block is contiguous
        ho = np.lexsort((local_row[halo], part[halo]))
        halo = halo[ho]
        ext_index = {int(g): len(owned[r]) + i for i, g in enumerate(halo)}
        sl = np.where(remote, 0, local_row[s])
        if remote.any():
            sl[remote] = np.array([ext_index[int(g)] for g in s[remote]])
        doms.append(Domain(r, world, owned[r], eids, halo, part[halo], local_row[halo], sl, dl))
    for r in range(world):
        d = doms[r]
        d.recv_counts = [int((d.halo_owner == p).sum()) for p in range(world)]
        d.send = [doms[p].halo_row[doms[p].halo_owner == r] for p in range(world)]
    return doms


def local_domain(part, rank, world, src_global, group=None):
    """This rank's :class:`Domain` from its own edges only (edges into the owned atoms, sorted
    by (owned row, source); ``src_global`` their global source ids), for graphs built per rank (the device radius
    graph over the owned atoms): no global edge list is formed.  Halo rows are ordered by
    (owner, owner row); the send lists come from one all-gather of the halo ids.  Returns the
    domain and the edges' sources in the extended [owned | halo] numbering (a tensor on the
    edges' device).  ``Domain.edges`` holds local edge ids (there are no global ones)."""
    import torch
    import torch.distributed as dist

    part = np.asarray(part)
    n = len(part)
    order = np.argsort(part, kind="stable")
    local_row = np.empty(n, dtype=np.int64)
    counts = np.bincount(part, minlength=world)
    starts = np.concatenate([[0], np.cumsum(counts)])
    for r in range(world):
        local_row[order[starts[r]:starts[r + 1]]] = np.arange(counts[r])
    owned = order[starts[rank]:starts[rank + 1]]  # sorted global ids (stable argsort)
    dev = src_global.device
    part_t = torch.as_tensor(part, device=dev)
    remote = part_t[src_global] != rank
    halo = torch.unique(src_global[remote]).cpu().numpy()
    halo = halo[np.lexsort((local_row[halo], part[halo]))]
    ext_map = torch.full((n,), -1, dtype=torch.long, device=dev)
    ext_map[torch.as_tensor(owned, device=dev)] = torch.arange(len(owned), device=dev)
    ext_map[torch.as_tensor(halo, device=dev)] = len(owned) + torch.arange(len(halo), device=dev)
    src_local = ext_map[src_global]
    halos = [halo]
    if world > 1:
        halos = [None] * world
        dist.all_gather_object(halos, halo, group=group)
    dom = Domain(rank, world, owned, np.arange(int(src_global.numel())), halo, part[halo], local_row[halo],
                 np.zeros(0, np.int64), np.zeros(0, np.int64))
    dom.recv_counts = [int((dom.halo_owner == p).sum()) for p in range(world)]
    dom.send = [local_row[h[part[h] == rank]] for h in halos]
    return dom, src_local
