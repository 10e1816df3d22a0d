"""Halo (ghost-node) exchange for graph-partitioned message passing.

Every Edgewise layer needs the features of its edges' source nodes; sources owned by other
ranks form this rank's halo.  :class:`HaloPlan` provides ``extend(x_node, graph)`` ->
``[owned rows | halo rows]`` with the matching backward (halo gradients are summed back into
the owners' rows).  Two transports:

* ``"collective"`` - ``all_to_all_single`` of the needed rows inside an autograd function
  (NCCL on GPUs, gloo on CPU).  This is the reference's design (``helm/nn/communication.py:
  190-340``) without its per-exchange device synchronise and global barrier.
* ``"peer"`` - owners publish their rows in a symmetric-memory staging buffer and the edge
  kernels load halo rows straight from the owner's buffer over NVLink; halo gradients are
  stored into the owner's receive slots and summed there (see :mod:`maloq_b200.parallel.peer_halo`).
"""

from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist


class _Exchange(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, plan):
        ctx.plan = plan
        return plan.fetch(x)

    @staticmethod
    def backward(ctx, g_halo):
        return ctx.plan.return_grads(g_halo), None


class HaloPlanError(RuntimeError):
    """The ranks' halo plans disagree (a rank expects rows that its owner will not send)."""


def validate_halo_plan(domain, group=None):
    """Check on the host, with one all-gather of the plan sizes, that every rank's receive
    count from each owner equals the number of rows that owner sends it, and that halo rows
    point inside their owner's rows.  Raises :class:`HaloPlanError` on every rank otherwise
    (a corrupted or stale plan would make the exchange read or write the wrong rows)."""
    world = domain.world
    if world == 1:
        return
    mine = {"recv": [int(c) for c in domain.recv_counts], "send": [int(len(s)) for s in domain.send],
            "n_own": int(domain.n_own), "max_row": {int(p): int(domain.halo_row[domain.halo_owner == p].max())
                                                    for p in set(domain.halo_owner.tolist())}}
    allp = [None] * world
    dist.all_gather_object(allp, mine, group=group)
    bad = []
    for q in range(world):
        for p in range(world):
            if allp[q]["recv"][p] != allp[p]["send"][q]:
                bad.append(f"rank {q} expects {allp[q]['recv'][p]} rows from rank {p}, which sends "
                           f"{allp[p]['send'][q]}")
        for p, mr in allp[q]["max_row"].items():
            if mr >= allp[p]["n_own"]:
                bad.append(f"rank {q} reads row {mr} of rank {p}, which owns {allp[p]['n_own']} rows")
    if bad:
        raise HaloPlanError("inconsistent halo plans: " + "; ".join(bad[:4]))


class HaloPlan:
    def __init__(self, domain, device, group=None, transport="collective", validate=True):
        self.domain = domain
        self.device = torch.device(device)
        self.group = group
        self.transport = transport
        self.world = domain.world
        self.n_own = domain.n_own
        self.n_halo = len(domain.halo)
        self.send_counts = [len(s) for s in domain.send]
        self.recv_counts = list(domain.recv_counts)
        cat = np.concatenate(domain.send) if sum(self.send_counts) else np.zeros(0, dtype=np.int64)
        self.send_idx = torch.as_tensor(cat, dtype=torch.long, device=self.device)
        self.peer = None
        if validate and dist.is_initialized():
            validate_halo_plan(domain, group)

    # ------------------------------------------------------------------ collective transport
    def fetch(self, x):
        rest = tuple(x.shape[1:])
        send = x.index_select(0, self.send_idx).contiguous()
        recv = x.new_empty((self.n_halo,) + rest)
        if self.world > 1:
            dist.all_to_all_single(recv, send, self.recv_counts, self.send_counts, group=self.group)
        return recv

    def return_grads(self, g_halo):
        rest = tuple(g_halo.shape[1:])
        g_halo = g_halo.contiguous()
        back = g_halo.new_empty((int(self.send_idx.numel()),) + rest)
        if self.world > 1:
            dist.all_to_all_single(back, g_halo, self.send_counts, self.recv_counts, group=self.group)
        gx = g_halo.new_zeros((self.n_own,) + rest)
        gx.index_add_(0, self.send_idx, back)
        return gx

    def gather_halo(self, x):
        return _Exchange.apply(x, self)

    def extend(self, x_node, graph=None):
        """[owned | halo] rows, differentiable (collective transport; the peer transport is used
        inside the fused edge kernels instead)."""
        if self.world == 1:
            return x_node
        # every rank joins the exchange: a rank without halo rows may still send rows
        return torch.cat([x_node, self.gather_halo(x_node)], dim=0)

    def materialize(self, x_node):
        """[owned | halo] rows as one differentiable local tensor with either transport (used
        by chunked execution, where the chunks share one exchange per layer)."""
        if self.world == 1:
            return x_node
        if self.transport == "peer":
            return self.peer_for(tuple(x_node.shape[1:])).fetch(x_node.contiguous().float())
        return self.extend(x_node)

    def peer_for(self, row_shape, n_slots=32):
        """The NVLink halo (created on first use - a collective step on every rank)."""
        if self.peer is None:
            from .peer_halo import PeerHalo

            self.peer = PeerHalo(self.domain, self.device, row_shape, n_slots=n_slots, group=self.group)
        return self.peer

    def gather_source(self, x_node, graph):
        """Features of every local edge's source node (reference-op path)."""
        return self.extend(x_node, graph).index_select(0, graph.src)


def partition_batch(sample, domain, pair_table=None, device="cpu", transport="collective", group=None,
                    target_dtype=torch.float32):
    """The GraphBatch of one rank for a partitioned structure ``sample`` (a GraphSample with
    global numbering).  Targets, if present, are restricted to owned nodes / local edges."""
    from ..data.batch import GraphBatch
    from ..data.graph import dst_pointer

    z = sample.z
    own = domain.owned
    e = domain.edges
    src_g, dst_g = sample.src[e], sample.dst[e]
    kw = dict(
        atomic_numbers=torch.as_tensor(z[own]),
        pos=torch.as_tensor(sample.pos[own], dtype=torch.float32),
        atom_charge=torch.as_tensor(sample.atom_charge[own]) if getattr(sample, "atom_charge", None) is not None
        else torch.full((len(own),), sample.charge, dtype=torch.long),
        atom_spin=torch.as_tensor(sample.atom_spin[own]) if getattr(sample, "atom_spin", None) is not None
        else torch.full((len(own),), sample.spin, dtype=torch.long),
        batch=torch.zeros(len(own), dtype=torch.long),
        edge_index=torch.as_tensor(np.stack([domain.src_local, domain.dst_local])),
        edge_attr=torch.as_tensor(sample.edge_attr[e], dtype=torch.float32),
        dst_ptr=torch.as_tensor(dst_pointer(domain.dst_local, len(own))),
        src_z=torch.as_tensor(z[src_g]),
        dst_z=torch.as_tensor(z[dst_g]),
        num_atoms_in_molecule=torch.as_tensor([len(own)]),
        global_node_ids=torch.as_tensor(own),
        global_edge_ids=torch.as_tensor(e),
    )
    b = GraphBatch(**kw)
    b.dst_ptr_host = kw["dst_ptr"].numpy()  # a host copy (not moved with the batch) for chunking
    if getattr(sample, "atom_mol_id", None) is not None:  # molecule of each owned atom (supergraphs)
        b.atom_mol_id = torch.as_tensor(sample.atom_mol_id[own])
    if pair_table is not None:
        b.node_pair_type = torch.as_tensor(pair_table.pair_type(z[own], z[own]))
        b.edge_pair_type = torch.as_tensor(pair_table.pair_type(z[src_g], z[dst_g]))
    if sample.node_y is not None:
        b.node_y = torch.as_tensor(sample.node_y)[:, own].to(target_dtype)
        b.y = torch.as_tensor(sample.y)[:, e].to(target_dtype)
    b = b.to(device)
    b.halo = HaloPlan(domain, device, group=group, transport=transport)
    b.num_nodes_ext = domain.n_ext
    return b


def local_batch(z, pos, dom, src_local, dst_local, vec, dst_ptr, pair_table=None, device="cuda",
                transport="peer", group=None, charge=0, spin=1):
    """The GraphBatch of one rank from its own edges (device tensors from the device radius
    graph: ``src_local`` in the [owned | halo] numbering of ``dom``, ``dst_local`` owned rows,
    ``vec = pos[src] - pos[dst]``, ``dst_ptr``), without any global edge list."""
    from ..data.batch import GraphBatch

    dev = torch.device(device)
    own_t = torch.as_tensor(dom.owned, device=dev)
    ext_t = torch.as_tensor(np.concatenate([dom.owned, dom.halo]), device=dev)
    z_t = torch.as_tensor(np.asarray(z), device=dev)
    n_own = dom.n_own
    src_g = ext_t[src_local]
    vec = vec.to(dev)
    edge_attr = torch.cat([vec.norm(dim=1, keepdim=True), vec], 1).float()
    z_own = z_t[own_t]
    b = GraphBatch(
        atomic_numbers=z_own, pos=torch.as_tensor(np.asarray(pos)[dom.owned], dtype=torch.float32, device=dev),
        atom_charge=torch.full((n_own,), charge, dtype=torch.long, device=dev),
        atom_spin=torch.full((n_own,), spin, dtype=torch.long, device=dev),
        batch=torch.zeros(n_own, dtype=torch.long, device=dev),
        edge_index=torch.stack([src_local.to(dev), dst_local.to(dev)]), edge_attr=edge_attr,
        dst_ptr=dst_ptr.to(dev), src_z=z_t[src_g], dst_z=z_own[dst_local.to(dev)],
        num_atoms_in_molecule=torch.tensor([n_own], device=dev), global_node_ids=own_t,
    )
    if pair_table is not None:
        zt = torch.as_tensor(pair_table.z_to_type, device=dev)
        nt = pair_table.n_types
        b.node_pair_type = zt[z_own] * nt + zt[z_own]
        b.edge_pair_type = zt[b.src_z] * nt + zt[b.dst_z]
    b.halo = HaloPlan(dom, dev, group=group, transport=transport)
    b.num_nodes_ext = dom.n_ext
    return b
