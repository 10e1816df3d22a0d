"""Fused NVLink halo for graph-partitioned message passing.

Forward: before an Edgewise layer every rank copies its owned rows into a staging slot of a
symmetric-memory buffer and passes a peer barrier; the gather kernel then loads each halo
source row directly from the owning rank's slot (``peers[owner] + row``) while it rotates the
message - the halo never exists as a separate exchanged tensor.

Backward: the gather-backward kernel stores each halo row's gradient straight into its owner's
receive buffer (double-buffered; ``begin_grads``), a barrier among the neighbours follows, and
each owner sums its own gradient rows and its received rows with one fixed-order segmented sum,
``node_reduce`` (``finish_grads``) - a reduce-scatter done inside the scatter stage.  The
chunked path, which materialises [owned | halo] rows once per layer, pushes its halo rows with
``halo_push`` instead (``reduce_grads``).

All waits are the bounded peer barriers of ``comm.cu``, among each rank's halo neighbours only
(the owners it reads from and the ranks that read from it), not all ranks.  Staging slots are kept for
``n_slots`` consecutive layers so the backward pass can re-read the forward rows.
Reference behaviour: ``helm/nn/communication.py:190-340`` (NCCL P2P with a device
synchronise and a global barrier per exchange).
"""

from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from ..ops.native import count_launches

SPIN_LIMIT = 1 << 28


def halo_neighbours(domain):
    """Ranks this rank exchanges halo rows with: the owners it reads from and the ranks that
    read from it (symmetric across the ranks' domains)."""
    return sorted({p for p in range(domain.world) if p != domain.rank and
                   (domain.recv_counts[p] > 0 or len(domain.send[p]) > 0)})


def _signed64(m):
    """A 64-bit member mask as the signed integer the binding takes."""
    return m - (1 << 64) if m >= 1 << 63 else m


class _PeerFetch(torch.autograd.Function):
    """[owned | halo] rows as one local tensor: publish, then copy every halo row out of its
    owner's staging slot (peer loads); backward returns the halo gradients to their owners."""

    @staticmethod
    def forward(ctx, x_node, peer):
        ctx.peer = peer
        slot = peer.publish(x_node)
        ext = x_node.new_empty((peer.n_own + peer.n_halo,) + peer.row_shape)
        ext[: peer.n_own] = x_node
        if peer.n_halo:
            peer.lib.halo_fetch(peer.table_ptr(slot), peer.halo_owner, peer.halo_row, ext[peer.n_own:])
            count_launches(1)
        return ext

    @staticmethod
    def backward(ctx, g):
        return ctx.peer.reduce_grads(g), None


class PeerHalo:
    def __init__(self, domain, device, row_shape, n_slots=16, group=None):
        import torch.distributed._symmetric_memory as symm_mem

        from ..ops.kernels import lib

        self.lib = lib()
        self.group = group or dist.group.WORLD
        self.device = torch.device(device)
        self.rank, self.world = domain.rank, domain.world
        self.row_shape = tuple(row_shape)
        self.sc = int(np.prod(row_shape))
        self.n_own = domain.n_own
        self.n_halo = len(domain.halo)
        self.n_slots = n_slots
        # halo counts of every rank by owner: counts[q][r] = rows rank q reads from rank r
        mine = torch.tensor(domain.recv_counts + [domain.n_own], dtype=torch.int64)
        allc = [torch.zeros_like(mine) for _ in range(self.world)]
        dist.all_gather_object(allc, mine, group=self.group)
        counts = np.stack([c.numpy()[: self.world] for c in allc])
        n_owns = [int(c.numpy()[self.world]) for c in allc]
        self.max_own = max(n_owns)
        recv_total = counts.sum(axis=0)  # rows each rank receives
        self.max_recv = int(max(1, recv_total.max()))
        # symmetric buffers: staging slots and two receive buffers
        self.stage = symm_mem.empty(n_slots * self.max_own * self.sc, dtype=torch.float32, device=self.device)
        self.hdl = symm_mem.rendezvous(self.stage, self.group.group_name)
        self.recvbuf = symm_mem.empty(2 * self.max_recv * self.sc, dtype=torch.float32, device=self.device)
        self.hdl_r = symm_mem.rendezvous(self.recvbuf, self.group.group_name)
        slot_bytes = self.max_own * self.sc * 4
        bases = np.array(self.hdl.buffer_ptrs, dtype=np.int64)
        self.tables = torch.tensor(np.stack([bases + k * slot_bytes for k in range(n_slots)]), dtype=torch.int64,
                                   device=self.device)
        rb = np.array(self.hdl_r.buffer_ptrs, dtype=np.int64)
        self.recv_tables = torch.tensor(np.stack([rb + k * self.max_recv * self.sc * 4 for k in range(2)]),
                                        dtype=torch.int64, device=self.device)
        self.pads = torch.tensor(self.hdl.signal_pad_ptrs, dtype=torch.int64, device=self.device)
        self.halo_owner = torch.as_tensor(domain.halo_owner.astype(np.int32), device=self.device)
        self.halo_row = torch.as_tensor(domain.halo_row.astype(np.int64), device=self.device)
        # where my halo rows land in their owners' receive buffers
        slot = np.zeros(self.n_halo, dtype=np.int64)
        for r in range(self.world):
            sel = np.flatnonzero(domain.halo_owner == r)
            off = int(counts[: self.rank, r].sum())
            slot[sel] = off + np.arange(len(sel))
        self.recv_slot = torch.as_tensor(slot, device=self.device)
        # owner side: received rows -> my local rows, as a CSR for a fixed-order sum
        send_idx = np.concatenate(domain.send) if sum(len(s) for s in domain.send) else np.zeros(0, np.int64)
        self.n_recv = len(send_idx)
        perm = np.argsort(send_idx, kind="stable")
        ptr = np.concatenate([[0], np.cumsum(np.bincount(send_idx, minlength=self.n_own))])
        self.recv_perm = torch.as_tensor(perm.astype(np.int64), device=self.device)
        self.recv_ptr = torch.as_tensor(ptr.astype(np.int64), device=self.device)
        # each owned row is its own single "edge" in the destination walk of node_reduce, so the
        # reduction adds the owned gradient and the received halo rows in one pass
        self.self_ptr = torch.arange(self.n_own + 1, dtype=torch.int64, device=self.device)
        # halo neighbours: the owners I read from and the ranks that read from me (a symmetric
        # relation); the peer barriers include only them (every rank calls them equally often,
        # so the epochs stay in step)
        self.neighbours = halo_neighbours(domain)
        self.mask = sum(1 << p for p in self.neighbours) | (1 << self.rank) if self.world <= 64 else 0
        self.epoch = 0
        self.next_slot = 0
        self.grad_calls = 0
        self.hdl.barrier()
        self.hdl_r.barrier()

    def _barrier(self):
        self.epoch += 1
        if self.mask:
            self.lib.peer_barrier_mask(self.pads.data_ptr(), self.rank, self.world, self.epoch, 0, SPIN_LIMIT,
                                       _signed64(self.mask))
        else:
            self.lib.peer_barrier(self.pads.data_ptr(), self.rank, self.world, self.epoch, 0, SPIN_LIMIT)
        count_launches(1)

    def table_ptr(self, slot):
        return self.tables[slot].data_ptr()

    def publish(self, x_node):
        """Copy the owned rows into the next staging slot and wait until every rank has."""
        slot = self.next_slot
        self.next_slot = (slot + 1) % self.n_slots
        view = self.stage[slot * self.max_own * self.sc: slot * self.max_own * self.sc + self.n_own * self.sc]
        view.view(self.n_own, *self.row_shape).copy_(x_node.detach())
        self._barrier()
        return slot

    def fetch(self, x_node):
        """Differentiable [owned | halo] rows (one publish, one peer copy per call)."""
        return _PeerFetch.apply(x_node, self)

    def begin_grads(self):
        """(receive-buffer index, its address table) for a backward kernel that stores the halo
        rows' gradients straight into their owners' receive slots (``recv_slot``)."""
        b = self.grad_calls % 2
        self.grad_calls += 1
        return b, self.recv_tables[b].data_ptr()

    def finish_grads(self, own, b):
        """After such a kernel: wait until the neighbours have stored their rows, then sum the
        owned gradient rows and the received ones (one fixed-order pass)."""
        self._barrier()
        own = own.contiguous()
        if self.n_recv == 0:
            return own
        recv = self.recvbuf[b * self.max_recv * self.sc:(b * self.max_recv + self.n_recv) * self.sc]
        out = torch.empty_like(own)
        self.lib.node_reduce(own.reshape(self.n_own, self.sc), self.self_ptr, recv.view(self.n_recv, self.sc),
                             self.recv_perm, self.recv_ptr, out.view(self.n_own, self.sc))
        count_launches(1)
        return out

    def reduce_grads(self, dx_ext):
        """Gradient of the extended rows -> gradient of the owned rows (halo rows summed on
        their owners)."""
        b = self.grad_calls % 2
        self.grad_calls += 1
        dx_ext = dx_ext.contiguous()
        halo = dx_ext[self.n_own:].reshape(self.n_halo, self.sc)
        if self.n_halo:
            self.lib.halo_push(halo, self.recv_tables[b].data_ptr(), self.halo_owner, self.recv_slot)
            count_launches(1)
        self._barrier()
        own = dx_ext[: self.n_own].reshape(self.n_own, *self.row_shape)
        if self.n_recv == 0:
            return own.clone()
        recv = self.recvbuf[b * self.max_recv * self.sc:(b * self.max_recv + self.n_recv) * self.sc]
        out = torch.empty_like(own)
        self.lib.node_reduce(own.reshape(self.n_own, self.sc), self.self_ptr, recv.view(self.n_recv, self.sc),
                             self.recv_perm, self.recv_ptr, out.view(self.n_own, self.sc))
        count_launches(1)
        return out
