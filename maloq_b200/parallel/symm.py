"""Fused gradient all-reduce over NVLink peer memory (no NCCL on the hot path).

The data-parallel gradient buckets live in one symmetric-memory allocation
(``torch.distributed._symmetric_memory``), so every rank can address every peer's buckets.
Reducing a bucket is two kernels on the reduction stream: ``peer_barrier(epoch)`` (one
CTA: every rank raises its epoch flag in every peer's signal pad and waits until all peers
raised theirs - the bucket is complete everywhere), then ``allreduce_multimem`` (NVLink SHARP
through NVSwitch, when the group supports multicast) or ``allreduce_p2p`` (peer
loads/stores): rank r reduces chunk r over all ranks, scales by 1/world and writes the result
into chunk r of every rank's bucket.  One more ``peer_barrier`` after the step's last bucket
(:meth:`PeerAllReduce.wait`) guarantees every chunk has been written everywhere before any
rank reads its gradients or reuses the buffer.

The reference reduces every parameter with its own synchronous NCCL all-reduce after
backward (``train_utils/splittrainer.py:204-218``).  Waits are bounded (see comm.cu); a
missing peer shows up as a non-zero ``error_status()`` instead of a hang.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops.native import count_launches

SPIN_LIMIT = 1 << 28  # polls of ~64 ns back-off: tens of seconds before a barrier gives up


class PeerAllReduce:
    def __init__(self, numel, device, group=None, use_multimem=None):
        import torch.distributed._symmetric_memory as symm_mem

        from ..ops.kernels import lib

        self.lib = lib()
        self.group = group or dist.group.WORLD
        self.device = torch.device(device)
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        self.buf = symm_mem.empty(max(4, (numel + 3) // 4 * 4), dtype=torch.float32, device=self.device)
        self.buf.zero_()
        name = self.group.group_name
        self.hdl = symm_mem.rendezvous(self.buf, name)
        self.bufs_dev = torch.tensor(self.hdl.buffer_ptrs, dtype=torch.int64, device=self.device)
        self.pads_dev = torch.tensor(self.hdl.signal_pad_ptrs, dtype=torch.int64, device=self.device)
        try:
            mc = int(self.hdl.multicast_ptr or 0)
        except Exception:  # noqa: BLE001 - no multicast object for this group
            mc = 0
        if use_multimem is None:
            # NVLS moves 1.5x the bucket per GPU in each direction at two ranks (the switch reads
            # both copies and writes both); peer loads/stores move 1x, so two ranks use p2p
            use_multimem = self.world > 2
        self.mc = mc if use_multimem else 0
        self.epoch = 0
        self.pending = None
        self.hdl.barrier()

    @property
    def transport(self):
        return "multimem" if self.mc else "p2p"

    def view(self, offset, numel):
        return self.buf[offset:offset + numel]

    def _barrier(self):
        self.epoch += 1
        self.lib.peer_barrier(self.pads_dev.data_ptr(), self.rank, self.world,
                              self.epoch, 0, SPIN_LIMIT)
        count_launches(1)

    def all_reduce_(self, flat, side_stream=None, scale=1.0):
        """Reduce ``flat`` (a view of this object's buffer) in place: sum over ranks * scale."""
        off = flat.data_ptr() - self.buf.data_ptr()
        assert off % 16 == 0 and 0 <= off and flat.is_contiguous(), "bucket must be an aligned view of the buffer"
        off //= 4
        n = flat.numel()
        if self.device.type != "cuda":  # host memory (tests): in order, no streams
            self._reduce(off, n, scale)
            self.pending = "host"
            return
        stream = side_stream or torch.cuda.current_stream(self.device)
        if side_stream is not None:
            side_stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(stream):
            self._reduce(off, n, scale)
            self.pending = stream

    def _reduce(self, off, n, scale):
        self._barrier()
        if self.mc:
            self.lib.allreduce_multimem(self.mc, self.rank, self.world, off, n, scale)
        else:
            self.lib.allreduce_p2p(self.bufs_dev.data_ptr(), self.rank, self.world, off, n, scale)
        count_launches(1)

    def wait(self, stream):
        """Close the step: one peer barrier after the last bucket (on the reduction stream),
        then ``stream`` waits for it."""
        side = getattr(self, "pending", None)
        if side is None:
            return
        if side == "host":
            self._barrier()
            self.pending = None
            return
        with torch.cuda.stream(side):
            self._barrier()
            ev = torch.cuda.Event()
            ev.record(side)
        stream.wait_event(ev)
        self.pending = None
