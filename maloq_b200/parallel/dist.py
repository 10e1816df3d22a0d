"""Process-group bootstrap and teardown (reference ``train_utils/utils_compute.py:14-132``).

One process per GPU.  Rank/world come from ``RANK``/``WORLD_SIZE`` (torchrun) or
``SLURM_PROCID``/``SLURM_NTASKS``; the local GPU from ``LOCAL_RANK``/``SLURM_LOCALID``.
A single process without a launcher gets a world of one on ``tcp://127.0.0.1``.
"""

from __future__ import annotations

import atexit
import datetime
import os

import torch
import torch.distributed as dist


def env_rank_world():
    rank = int(os.environ.get("RANK", os.environ.get("SLURM_PROCID", 0)))
    world = int(os.environ.get("WORLD_SIZE", os.environ.get("SLURM_NTASKS", 1)))
    local = int(os.environ.get("LOCAL_RANK", os.environ.get("SLURM_LOCALID", rank)))
    return rank, world, local


def setup_env(rank=None, world_size=None, backend=None, timeout_s=600):
    """Initialise torch.distributed; returns the device of this rank."""
    r, w, local = env_rank_world()
    rank = r if rank is None else rank
    world_size = w if world_size is None else world_size
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    if torch.cuda.is_available():
        dev = torch.device("cuda", local % torch.cuda.device_count())
        torch.cuda.set_device(dev)
    else:
        dev = torch.device("cpu")
    os.environ.setdefault("TORCH_NCCL_ASYNC_ERROR_HANDLING", "1")
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29500")
        kw = dict(backend=backend, rank=rank, world_size=world_size,
                  timeout=datetime.timedelta(seconds=timeout_s))
        if backend == "nccl" and dev.type == "cuda":
            kw["device_id"] = dev
        dist.init_process_group(init_method="env://", **kw)
        atexit.register(cleanup_process_group)
    return dev


def cleanup_process_group(sync_barrier=False):
    """Best-effort teardown (safe to call twice, or when init never happened)."""
    try:
        if dist.is_available() and dist.is_initialized():
            if sync_barrier:
                try:
                    dist.barrier()
                except Exception:  # noqa: BLE001 - a dead peer must not block shutdown
                    pass
            dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        pass


def rank():
    return dist.get_rank() if dist.is_available() and dist.is_initialized() else 0


def world_size():
    return dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1


def split_indices(n_total, rank_, world, drop_remainder=True):
    """Contiguous shard of ``range(n_total)`` for this rank (``utils_compute.py:98-132``)."""
    per = n_total // world
    if drop_remainder:
        return list(range(rank_ * per, (rank_ + 1) * per))
    extra = n_total % world
    start = rank_ * per + min(rank_, extra)
    return list(range(start, start + per + (1 if rank_ < extra else 0)))
