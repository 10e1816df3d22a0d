"""Reference arm of ``bench.py``: the unmodified reference package (installed under
``baseline/_ref``) trained through its own public modules on the drug-like DP config.

Nothing from ``maloq_b200`` is imported here: the model is the reference's
``maloq.helm.esen_osh.eSEN_Backbone`` + ``Fock_Irreps_Head`` built the way its
``TrainingWorkflow.build_model`` builds them (``training_workflow.py:503-571``), the loss is
its ``rmse_mse_padded_loss`` (``train_utils/loss.py:27``), the optimizer ``torch.optim.Adam``,
and the data-parallel gradient sum its per-parameter NCCL all-reduce
(``splittrainer.py:204-218``).  The molecules are random drug-like chains of the config's
shape (30-50 atoms of H, C, N, O, F, S, Cl; 6 A graph) built with numpy here; the targets are
random label rows of the head's output width (throughput only).

The reference forces ``mmax = lmax`` (``training_workflow.py:511``); its Edgewise cannot run
with ``mmax < lmax``.  The arm therefore runs lmax = mmax = 4, which does more work per edge
than the config's mmax = 2, and says so in its JSON line.

Prints one JSON line (rank 0); exits 0 with an ``unavailable`` line when the package or one of
its run-time dependencies cannot be imported.
"""

from __future__ import annotations

import importlib
import importlib.util
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(HERE, "baseline", "_ref")
# run-time imports of the stock training path (esen_osh, esen_block, communication,
# fock_targets_batched, splittrainer, training_workflow)
DEPS = ["e3nn", "fairchem", "torch_geometric", "cupy", "mpi4py", "ase", "apsw", "h5py", "pyscf", "matplotlib"]
MODULES = ["maloq.helm.esen_osh", "maloq.train_utils.loss", "maloq.train_utils.training_workflow"]


def unavailable(why):
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)
    sys.exit(0)


def probe():
    """Import the reference's stock modules; on failure name every missing dependency."""
    if not os.path.isdir(os.path.join(REF, "maloq")):
        unavailable("baseline/_ref not installed (pip install --no-index --no-deps --target baseline/_ref "
                    "<copy of the reference>)")
    sys.path.insert(0, REF)
    missing = [d for d in DEPS if importlib.util.find_spec(d) is None]
    try:
        mods = [importlib.import_module(m) for m in MODULES]
    except Exception as e:  # noqa: BLE001 - any import failure ends the arm
        unavailable(f"reference package installed in baseline/_ref but does not import: {type(e).__name__}: {e}; "
                    f"missing offline: {', '.join(missing) or 'none'}")
    return mods


def molecule(rng, lo=30, hi=50):
    import numpy as np

    n = int(rng.integers(lo, hi + 1))
    z = rng.choice([1, 6, 7, 8, 9, 16, 17], size=n, p=[0.45, 0.35, 0.08, 0.08, 0.04 / 3, 0.04 / 3, 0.04 / 3])
    pos = np.zeros((n, 3))
    for i in range(1, n):
        d = rng.normal(size=3)
        pos[i] = pos[rng.integers(0, i)] + d / np.linalg.norm(d) * rng.uniform(1.0, 1.6)
    return z, pos


def main():
    esen, rloss, _ = probe()
    import numpy as np
    import torch
    import torch.distributed as dist

    steps = int(os.environ.get("BENCH_STEPS", "20"))
    warmup = int(os.environ.get("BENCH_WARMUP", "5"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1:
        dist.init_process_group("nccl")
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    from e3nn.o3 import Irreps

    lmax, C = 4, 128
    irreps_out = Irreps("+".join(f"1x{l}e" for l in range(lmax + 1)) * 1)
    backbone = esen.eSEN_Backbone(irreps_out, sphere_channels=C, hidden_channels=C, lmax=lmax, mmax=lmax, cutoff=6.0,
                                  edge_channels=C, num_layers=6, act_type="gate", mlp_type="spectral",
                                  num_distance_basis=128, include_edges=True).to(dev)
    head = esen.Fock_Irreps_Head(Irreps([(C, (l, 1)) for l in range(lmax + 1)]), irreps_out, lmax=lmax,
                                 sphere_channels=C, ls_list=[0, 1, 2]).to(dev)
    params = list(backbone.parameters()) + list(head.parameters())
    opt = torch.optim.Adam(params, lr=1e-4)

    class Batch(dict):
        __getattr__ = dict.__getitem__

    rng = np.random.default_rng(1000 + rank)
    zs, ps, srcs, dsts, vecs, counts, off = [], [], [], [], [], [], 0
    for _ in range(32):
        z, pos = molecule(rng)
        d = pos[:, None] - pos[None]
        r = np.linalg.norm(d, axis=-1)
        s, t = np.nonzero((r < 6.0) & (r > 0))
        srcs.append(s + off)
        dsts.append(t + off)
        vecs.append(np.concatenate([r[s, t, None], d[s, t]], 1))
        zs.append(z)
        ps.append(pos)
        counts.append(len(z))
        off += len(z)
    b = Batch(pos=torch.tensor(np.concatenate(ps), dtype=torch.float32, device=dev),
              edge_index=torch.tensor(np.stack([np.concatenate(srcs), np.concatenate(dsts)]), device=dev),
              edge_attr=torch.tensor(np.concatenate(vecs), dtype=torch.float32, device=dev),
              atomic_numbers=torch.tensor(np.concatenate(zs), device=dev),
              charge=torch.zeros(32, dtype=torch.long, device=dev),
              spin_multiplicity=torch.ones(32, dtype=torch.long, device=dev),
              num_atoms_in_molecule=torch.tensor(counts, device=dev))
    n_edges = b.edge_index.shape[1]

    def step():
        out = head(backbone(b), b)
        node_out, edge_out = out[0], out[1]
        loss = rloss.rmse_mse_padded_loss(node_out, torch.zeros_like(node_out)) + \
            rloss.rmse_mse_padded_loss(edge_out, torch.zeros_like(edge_out))
        opt.zero_grad(set_to_none=True)
        loss.backward()
        if world > 1:  # the reference's per-parameter all-reduce
            for p in params:
                if p.grad is not None:
                    dist.all_reduce(p.grad)
                    p.grad /= world
        opt.step()
        return loss

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        step()
    e.record()
    torch.cuda.synchronize()
    ms = torch.tensor([s.elapsed_time(e) / steps], device=dev, dtype=torch.float64)
    t0 = time.time()
    for _ in range(steps):
        step().item()
    e2e_ms = (time.time() - t0) * 1e3 / steps
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = ms.item()
    if rank == 0:
        print(json.dumps({
            "impl": "reference", "metric": "train graphs/s (drug-like DP, device-timed, max over ranks)",
            "value": round(32 * world / (ms / 1e3), 2), "unit": "graphs/s", "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp32", "data": "synthetic (random drug-like chains; random targets)",
            "config": {"model": "reference eSEN lmax=4 mmax=4 (the reference requires mmax=lmax) C=128 layers=6",
                       "global_batch": 32 * world, "edges_per_gpu_step": int(n_edges),
                       "parallelism": f"dp{world}"},
            "e2e": {"value": round(32 * world / (e2e_ms / 1e3), 2), "unit": "graphs/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 4}}), flush=True)


if __name__ == "__main__":
    main()
