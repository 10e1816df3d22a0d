"""Data-parallel gradient synchronisation, bucketed and overlapped with backward.

Reference behaviour (``splittrainer.py:204-218``): after ``loss.backward()`` every
parameter's gradient is all-reduced on its own, synchronously, then divided by the world
size.  :class:`GradSync` instead

* packs gradients into flat fp32 buckets (in reverse registration order, roughly the
  order backward produces them); each parameter's ``.grad`` is a view of its bucket, so
  autograd accumulates straight into the bucket with no copy;
* starts a bucket's reduction from a post-accumulate-grad hook as soon as its last
  gradient is written, on a side stream, while backward keeps running;
* reduces with one of three transports:

  - ``"fused"`` - the NVLink peer-memory all-reduce kernel of
    :mod:`maloq_b200.parallel.symm` (reduce + 1/world scale in one kernel, no NCCL);
  - ``"nccl"`` - ``all_reduce(AVG)`` per bucket (the NCCL baseline);
  - ``"per_param"`` - the reference's per-parameter reduction after backward.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


class _Bucket:
    def __init__(self, params, device, index, storage=None):
        self.params = params
        self.index = index
        n = sum(p.numel() for p in params)
        self.buf = storage if storage is not None else torch.zeros(n, dtype=torch.float32, device=device)
        self.views = []
        off = 0
        for p in params:
            self.views.append(self.buf[off:off + p.numel()].view_as(p))
            off += p.numel()
        self.pending = len(params)
        self.launched = False


class GradSync:
    def __init__(self, params, bucket_mb: float = 16.0, mode: str = "nccl", group=None):
        self.params = [p for p in params if p.requires_grad]
        self.mode, self.group = mode, group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        if any(p.dtype != torch.float32 for p in self.params):
            raise ValueError("GradSync keeps fp32 master gradients; parameters must be fp32")
        self.device = self.params[0].device if self.params else torch.device("cpu")
        self.is_cuda = self.device.type == "cuda"
        self.side = torch.cuda.Stream(device=self.device) if self.is_cuda else None
        limit = int(bucket_mb * 2**20 / 4)
        buckets, cur, size = [], [], 0
        for p in reversed(self.params):
            cur.append(p)
            size += p.numel()
            if size >= limit:
                buckets.append(cur)
                cur, size = [], 0
        if cur:
            buckets.append(cur)
        self._fused = None
        if mode == "fused" and self.world > 1:
            from .symm import PeerAllReduce

            sizes = [(sum(p.numel() for p in b) + 3) // 4 * 4 for b in buckets]
            self._fused = PeerAllReduce(sum(sizes), self.device, group)
            offs = [sum(sizes[:i]) for i in range(len(sizes))]
            self.buckets = [_Bucket(b, self.device, i, self._fused.view(o, sum(p.numel() for p in b)))
                            for i, (b, o) in enumerate(zip(buckets, offs))]
        else:
            self.buckets = [_Bucket(b, self.device, i) for i, b in enumerate(buckets)]
        self._owner = {}
        for b in self.buckets:
            for p, v in zip(b.params, b.views):
                self._owner[p] = (b, v)
        self.works = []
        if mode in ("nccl", "fused"):
            for p in self.params:
                p.register_post_accumulate_grad_hook(self._hook)

    # ------------------------------------------------------------------
    def begin_step(self):
        """Attach bucket views as ``.grad`` and zero the buckets (call before backward)."""
        for b in self.buckets:
            b.buf.zero_()
            b.pending = len(b.params)
            b.launched = False
            for p, v in zip(b.params, b.views):
                p.grad = v
        self.works = []

    def _hook(self, p):
        b, v = self._owner[p]
        if p.grad is not v:  # autograd replaced the view (e.g. grad set to None); copy back
            v.copy_(p.grad)
            p.grad = v
        b.pending -= 1
        if b.pending == 0:
            self._launch(b)

    def _launch(self, b):
        if b.launched or self.world == 1:
            b.launched = True
            return
        b.launched = True
        if self.mode == "fused":
            self._fused.all_reduce_(b.buf, side_stream=self.side, scale=1.0 / self.world)
            return
        if self.is_cuda:
            self.side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.side):
                self.works.append((dist.all_reduce(b.buf, op=dist.ReduceOp.AVG, group=self.group, async_op=True), None))
        else:
            self.works.append((dist.all_reduce(b.buf, op=dist.ReduceOp.SUM, group=self.group, async_op=True), b))

    def finish(self):
        """Make the current stream wait for every reduction (call after backward)."""
        if self.world == 1:
            return
        if self.mode == "per_param":
            for p in self.params:
                if p.grad is not None:
                    dist.all_reduce(p.grad, op=dist.ReduceOp.SUM, group=self.group)
                    p.grad /= self.world
            return
        for b in self.buckets:  # buckets whose parameters got no gradient this step
            if not b.launched:
                self._launch(b)
        if self.mode == "fused":
            self._fused.wait(torch.cuda.current_stream(self.device) if self.is_cuda else None)
            return
        for w, b in self.works:
            w.wait()
            if b is not None:
                b.buf /= self.world
        self.works = []
