"""Partitioned inference output: each rank writes the Hamiltonian blocks it owns.

The reference gathers every rank's outputs to every rank and rank 0 writes one matrix
(``train_utils/splittrainer.py:825-1148``, ``:1406-1532``).  Here rank r converts its node
and edge labels to blocks (``get_H`` + label->block scatter) and writes
``hamiltonian_rank{r}.npz`` with global atom indices, so nothing is gathered;
:func:`load_partitioned_hamiltonian` merges the shards into one block-sparse matrix.
"""

from __future__ import annotations

import glob
import os

import numpy as np
import torch

from ..data.labels import BlockSparseMatrix


def _global_ids(batch):
    own = batch.global_node_ids.cpu().numpy() if getattr(batch, "global_node_ids", None) is not None \
        else np.arange(batch.num_nodes)
    return own


def write_partition_hamiltonian(folder, batch, node_out, edge_out, labeler, partition=None, rank=None,
                                global_src=None, global_dst=None):
    """Write this rank's blocks; returns the path.  ``node_out``/``edge_out`` are coupled labels
    of the owned nodes / local edges.  Global edge endpoints come from ``global_src``/``global_dst``
    (or the batch's local numbering when the graph is not partitioned)."""
    import torch.distributed as dist

    rank = (dist.get_rank() if dist.is_initialized() else 0) if rank is None else rank
    os.makedirs(folder, exist_ok=True)
    own = _global_ids(batch)
    z_own = batch.atomic_numbers.cpu().numpy()
    if global_src is None:
        ei = batch.edge_index.cpu().numpy()
        halo = batch.halo.domain.halo if getattr(batch, "halo", None) is not None else np.zeros(0, np.int64)
        ext = np.concatenate([own, halo])
        gsrc, gdst = ext[ei[0]], own[ei[1]]
    else:
        gsrc, gdst = np.asarray(global_src), np.asarray(global_dst)
    rows = np.concatenate([gsrc, own])
    cols = np.concatenate([gdst, own])
    src_z = batch.src_z.cpu().numpy()
    dst_z = batch.dst_z.cpu().numpy()
    zr = np.concatenate([src_z, z_own])
    zc = np.concatenate([dst_z, z_own])
    tbl = labeler.table
    pt = torch.as_tensor(tbl.pair_type(zr, zc), device=labeler.device)
    nr, nc = tbl.norb[tbl.z_to_type[zr]], tbl.norb[tbl.z_to_type[zc]]
    ptr = np.concatenate([[0], np.cumsum(nr * nc)]).astype(np.int64)
    coupled = torch.cat([edge_out, node_out], 0).to(labeler.device, labeler.dtype)
    from ..ops import labels as lab

    data = lab.coupled_to_blocks(coupled, torch.as_tensor(ptr, device=labeler.device), pt, labeler.pos_t,
                                 labeler.transform, int(ptr[-1]))
    path = os.path.join(folder, f"hamiltonian_rank{rank}.npz")
    np.savez(path, rows=rows, cols=cols, block_ptr=ptr, data=data.detach().float().cpu().numpy(),
             atom_ids=own, atom_z=z_own)
    return path


def load_partitioned_hamiltonian(folder, labeler, symmetrize=True) -> BlockSparseMatrix:
    """Merge every rank's shard into one block-sparse Hamiltonian (blocks sorted by (row, col));
    with ``symmetrize`` each block is replaced by (H_ij + H_ji^T) / 2."""
    shards = [np.load(p) for p in sorted(glob.glob(os.path.join(folder, "hamiltonian_rank*.npz")))]
    n = int(max(s["atom_ids"].max() for s in shards)) + 1
    z = np.zeros(n, dtype=np.int64)
    for s in shards:
        z[s["atom_ids"]] = s["atom_z"]
    rows = np.concatenate([s["rows"] for s in shards])
    cols = np.concatenate([s["cols"] for s in shards])
    blocks = []
    for s in shards:
        for b in range(len(s["rows"])):
            blocks.append(s["data"][s["block_ptr"][b]:s["block_ptr"][b + 1]])
    order = np.lexsort((cols, rows))
    tbl = labeler.table
    norb = tbl.norb[tbl.z_to_type[z]]
    orb_ptr = np.concatenate([[0], np.cumsum(norb)]).astype(np.int64)
    rows, cols = rows[order], cols[order]
    blocks = [blocks[i] for i in order]
    if symmetrize:
        key = {(int(r), int(c)): i for i, (r, c) in enumerate(zip(rows, cols))}
        sym = []
        for i, (r, c) in enumerate(zip(rows, cols)):
            a = blocks[i].reshape(norb[r], norb[c])
            j = key.get((int(c), int(r)))
            if j is not None:
                a = 0.5 * (a + blocks[j].reshape(norb[c], norb[r]).T)
            sym.append(a.ravel())
        blocks = sym
    ptr = np.concatenate([[0], np.cumsum([len(b) for b in blocks])]).astype(np.int64)
    return BlockSparseMatrix(rows, cols, ptr, np.concatenate(blocks) if blocks else np.zeros(0), orb_ptr)


@torch.no_grad()
def hamiltonian_shard(head, emb, batch, labeler, spin=0, out=None):
    """This rank's block-sparse Hamiltonian on the device, streamed: the edge blocks are made
    chunk by chunk (head -> coupled labels -> fused CG transform + scatter into the block data,
    ``coupled_to_blocks``), then the owned atoms' diagonal blocks, so no [E, D] label tensor is
    formed.  Block order: local edges (dst-sorted), then owned atoms.  Returns
    (data [n_data] fp32, block_ptr [n_blocks + 1] int64) on the device; ``out`` reuses a data
    buffer of the right size."""
    from ..ops import labels as lab

    dev = batch.atomic_numbers.device
    tbl = labeler.table
    zt = torch.as_tensor(tbl.z_to_type, device=dev)
    norb = torch.as_tensor(tbl.norb, device=dev)
    n_src = norb[zt[batch.src_z]]
    n_dst = norb[zt[batch.dst_z]]
    n_at = norb[zt[batch.atomic_numbers]]
    sizes = torch.cat([n_src * n_dst, n_at * n_at])
    ptr = torch.zeros(sizes.numel() + 1, dtype=torch.long, device=dev)
    ptr[1:] = torch.cumsum(sizes, 0)
    n_data = int(ptr[-1])
    data = out if out is not None and out.numel() == n_data else torch.empty(n_data, device=dev)
    E = batch.num_edges
    pos_t, T = labeler.pos_t.to(dev), labeler.transform
    chunks = emb.get("edge_chunks") or [(0, E)]
    edge_emb = emb["edge_embeddings"]
    node_dtype = emb["node_embeddings"].dtype
    for e0, e1 in chunks:
        lbl = head.edge_labels(edge_emb[e0:e1].to(node_dtype), spin)
        lab.coupled_to_blocks(lbl, ptr[e0:e1 + 1], batch.edge_pair_type[e0:e1], pos_t, T, n_data, out=data)
    nl = head.node_labels(emb["node_embeddings"], spin)
    lab.coupled_to_blocks(nl, ptr[E:], batch.node_pair_type, pos_t, T, n_data, out=data)
    return data, ptr
