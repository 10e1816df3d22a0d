"""NVLink communication paths of this library against their rooflines (one process per GPU).

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m maloq_b200.parallel.commbench [--mib 256]

* fused gradient all-reduce (``PeerAllReduce``: bounded peer barrier, peer-load or NVLS
  ``multimem`` reduction, barrier) and ``torch.distributed.all_reduce`` (NCCL) on the same
  fp32 buffer: bus bandwidth = bytes * 2 (N - 1) / N / time, the NVLink traffic per GPU of an
  all-reduce;
* halo fetch (``PeerHalo.fetch``: owned rows copied into the staging slot, peer barrier, halo
  rows loaded from the owner's slot over NVLink): each rank reads ``--halo-rows`` rows of
  (L+1)^2 x C fp32 from its neighbour; NVLink bytes = rows x row bytes.

Each figure is also given as a fraction of the per-direction NVLink copy bandwidth
``--link-gbs`` (770 GB/s measured on this hardware; 900 nominal).  Times are CUDA events on the
launching stream after warm-up, max over ranks; rank 0 prints one JSON line per path.
"""

from __future__ import annotations

import argparse
import json

import numpy as np
import torch
import torch.distributed as dist


def _timed(fn, iters, warm=3):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    t = torch.tensor([s.elapsed_time(e) / iters], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()  # ms


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--mib", type=int, nargs="+", default=[16, 256], help="all-reduce buffer sizes (MiB, fp32)")
    ap.add_argument("--halo-rows", type=int, default=20000)
    ap.add_argument("--own-rows", type=int, default=20000)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--link-gbs", type=float, default=770.0)
    a = ap.parse_args(argv)

    from . import dist as pdist
    from .partition import Domain
    from .peer_halo import PeerHalo
    from .symm import PeerAllReduce

    dev = pdist.setup_env(backend="nccl")
    rank, world = dist.get_rank(), dist.get_world_size()
    out = []

    # ---- all-reduce: fused (multimem where the group has a multicast object, and p2p) vs NCCL
    correct = True
    for mib in a.mib:
        n = mib * 2**20 // 4
        nbytes = n * 4
        for use_mm in (True, False):
            par = PeerAllReduce(n, dev, use_multimem=use_mm)
            if use_mm and not par.mc:
                continue
            buf = par.view(0, n)
            buf.fill_(1.0)

            def one():
                par.all_reduce_(buf)
                par.wait(torch.cuda.current_stream())

            ms = _timed(one, a.iters)
            bus = nbytes * 2 * (world - 1) / world / (ms * 1e-3) / 1e9
            out.append({"path": f"fused all-reduce ({par.transport})", "bytes": nbytes, "ms": round(ms, 4),
                        "bus_gbs": round(bus, 1), "frac_of_link": round(bus / a.link_gbs, 3)})
            correct &= bool(torch.allclose(buf[:1024], torch.full((1024,), float(world) ** (3 + a.iters),
                                                                    device=dev)))
            del par, buf
        t = torch.ones(n, device=dev)
        ms = _timed(lambda: dist.all_reduce(t), a.iters)
        bus = nbytes * 2 * (world - 1) / world / (ms * 1e-3) / 1e9
        out.append({"path": "NCCL all_reduce", "bytes": nbytes, "ms": round(ms, 4), "bus_gbs": round(bus, 1),
                    "frac_of_link": round(bus / a.link_gbs, 3)})
        del t

    # ---- halo fetch: rank r reads rows 0..H-1 of rank (r+1) % N
    M, H = a.own_rows, a.halo_rows
    nxt, prv = (rank + 1) % world, (rank - 1) % world
    dom = Domain(rank, world, np.arange(M) + rank * M, np.zeros(0, np.int64), np.arange(H) + nxt * M,
                 np.full(H, nxt), np.arange(H), np.zeros(0, np.int64), np.zeros(0, np.int64))
    dom.recv_counts = [H if p == nxt else 0 for p in range(world)]
    dom.send = [np.arange(H) if p == prv else np.zeros(0, np.int64) for p in range(world)]
    row = (25, 128)
    halo = PeerHalo(dom, dev, row)
    x = torch.randn(M, *row, device=dev) + rank
    with torch.no_grad():
        ms = _timed(lambda: halo.fetch(x), a.iters)
        ext = halo.fetch(x)
    torch.cuda.synchronize()
    hb = H * int(np.prod(row)) * 4
    gbs = hb / (ms * 1e-3) / 1e9
    out.append({"path": "halo fetch (publish + peer barrier + peer loads)", "halo_bytes": hb, "ms": round(ms, 4),
                "halo_gbs": round(gbs, 1), "frac_of_link": round(gbs / a.link_gbs, 3)})
    # the fetched rows are the neighbour's first rows (its x = randn + nxt: check the mean shift)
    ok_halo = abs(ext[M:].mean().item() - nxt) < 0.05
    if rank == 0:
        for o in out:
            o.update(n_gpus=world)
            print(json.dumps(o), flush=True)
        print(json.dumps({"checks": {"allreduce_sum": correct, "halo_rows_from_neighbour": bool(ok_halo)}}))
    pdist.cleanup_process_group()


if __name__ == "__main__":
    main()
