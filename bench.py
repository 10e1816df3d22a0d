"""Headline benchmark: training graphs/s on the drug-like data-parallel config.

Config (drug-like molecules, data-parallel bf16 on 1/2/4/8 B200): 30-50 atom
molecules from {H,C,N,O,F,S,Cl}, def2-SVP-like basis (H 5, 2nd row 14, S/Cl 18 orbitals,
labels of 324 entries, lmax 4), eSEN backbone lmax=4, mmax=2, 128 channels, 6 layers,
6 A graph cutoff, 32 molecules per GPU, Fock head with node reductions, rmse+mse loss,
Adam.  Weak scaling: every rank trains on its own 32 molecules per step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|torch|reference]

``native`` runs this framework's kernels; ``torch`` the same model on PyTorch ops with an
NCCL bucketed all-reduce (the reference-math baseline); ``reference`` the unmodified
reference package from ``baseline/_ref`` (prints an ``unavailable`` line when it cannot
be imported).  Rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
BASELINE_VALUE = None  # the reference publishes no number for this metric
METRIC = "train graphs/s (drug-like DP, device-timed, max over ranks)"
PARTITIONED = {
    # name: (dataset kind, default atoms, mmax, layers, what)
    "sio2": ("sio2", 20000, 2, 6, "train"),
    "slab": ("slab", 1_000_000, 2, 6, "infer"),
}
CONFIGS = {
    # name: (dataset kind, mmax, default layers, molecules per batch or None, atoms per batch cap)
    "druglike": ("druglike", 2, 6, 32, None),
    "large": ("large", 2, 8, None, 4096),
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="native", choices=["native", "torch", "reference"])
    ap.add_argument("--batch", type=int, default=32, help="molecules per GPU")
    ap.add_argument("--layers", type=int, default=6)
    ap.add_argument("--channels", type=int, default=128)
    ap.add_argument("--n-batches", type=int, default=4, help="distinct batches cycled per rank")
    ap.add_argument("--grad-sync", default=None)
    ap.add_argument("--atoms", type=int, default=None, help="atoms of the partitioned structure")
    ap.add_argument("--edge-chunk", type=int, default=131072,
                    help="partitioned configs: edges per chunk of the chunked (recomputed) block execution")
    ap.add_argument("--breakdown", action="store_true",
                    help="instead of the bench line: per-kernel-class device time of the training step "
                         "(torch profiler / CUPTI over --steps steps; shares, not a bench number)")
    ap.add_argument("--config", default="druglike", choices=list(CONFIGS) + list(PARTITIONED) + ["cpu"],
                    help="druglike (headline) or large (10-150 atoms, lmax 6, 8 layers, <=4096 atoms/GPU)")
    return ap.parse_args()


def labeler_name(kind):
    return {"druglike": "def2-SVP-like", "large": "def2-TZVP-like"}.get(kind, kind)


def reference_arm(args):
    """Run the unmodified reference through its public modules (``bench_reference.py``, which
    imports nothing from this framework).  Its JSON line (or ``unavailable`` line naming the
    missing modules) is printed as is."""
    env = dict(os.environ, BENCH_STEPS=str(args.steps), BENCH_WARMUP=str(args.warmup))
    r = subprocess.run([sys.executable, os.path.join(HERE, "bench_reference.py")], env=env, capture_output=True,
                       text=True)
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    if lines:
        return json.loads(lines[-1])
    if int(os.environ.get("RANK", "0")) != 0:
        return None
    last = (r.stderr.strip().splitlines() or ["no output"])[-1]
    return {"impl": "reference", "unavailable": f"reference run failed (rc {r.returncode}): {last}"}


class ClockSampler:
    def __init__(self, index):
        self.index, self.proc, self.path = index, None, f"/tmp/maloq_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}",
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 7:
                continue
            try:
                sm.append(float(f[0]))
                mx = float(f[1])
            except ValueError:
                continue
            for n, v in zip(names, f[3:7]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def timed_steps(args, device, world, step_resident, step_e2e):
    """Warm-up, then ``args.steps`` device-timed steps on resident inputs (L2 flushed before each
    step, outside its events), then ``args.steps`` end-to-end steps whose inputs are copied from
    pinned host memory and whose loss is read back each step.  Returns (device ms summed over
    steps, e2e ms, kernel launches in the device-timed region, clock record, losses) with both
    times the max over ranks."""
    import torch
    import torch.distributed as dist

    from maloq_b200 import ops

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    flush = torch.empty(256 * 2**20, dtype=torch.uint8, device=device)
    for i in range(args.warmup):
        step_resident(i)
    barrier()
    clocks = ClockSampler(device.index)
    clocks.start()
    launches0 = ops.launch_count()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    for i in range(args.steps):
        flush.zero_()
        ev[i][0].record()
        step_resident(i)
        ev[i][1].record()
    barrier()
    launches = ops.launch_count() - launches0
    ms = sum(a.elapsed_time(b) for a, b in ev)
    e2e_start, e2e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e2e_start.record()
    loss_vals = []
    for i in range(args.steps):
        _, _, loss = step_e2e(i)
        loss_vals.append(loss.item())
    e2e_end.record()
    barrier()
    clk = clocks.stop()
    t = torch.tensor([ms, e2e_start.elapsed_time(e2e_end)], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms = t.tolist()
    return ms, e2e_ms, launches, clk, loss_vals


KERNEL_CLASSES = [
    # (class, substrings of the kernel name)
    ("GEMM (tcgen05)", ("gemm_tc",)),
    ("split-K reduce", ("splitk_reduce",)),
    ("gather+rotate fwd/bwd", ("gather_rotate",)),
    ("rotate-back / rotate-grad", ("rotate_back", "rotate_grad")),
    ("node reduce", ("node_reduce",)),
    ("SO(2) gate", ("gate_fwd", "gate_bwd")),
    ("norms / atomwise gate / LN+SiLU", ("rms_norm", "ln_silu", "gate_l", "layernorm")),
    ("edge rotation", ("edge_rotation",)),
    ("loss", ("fock_loss",)),
    ("labels / head", ("basis_rows", "head_")),
    ("optimizer (Adam)", ("adam", "Adam")),
    ("copies / casts", ("copy", "Copy", "cat", "Cat", "memcpy", "Memcpy", "memset", "Memset")),
]


def step_breakdown(args, step, n_edges, n_nodes):
    """Device time of the training step split by kernel class, from the CUDA activity trace of
    ``args.steps`` steps (after ``args.warmup``).  The step's own CUDA-event time is taken in a
    separate, unprofiled pass, so 'idle' = event time - summed kernel time (the step runs on one
    stream).  Prints a markdown table and one JSON line."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(args.steps):
        step(i)
    e.record()
    torch.cuda.synchronize()
    ev_ms = s.elapsed_time(e) / args.steps
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for i in range(args.steps):
            step(i)
        torch.cuda.synchronize()
    per_kernel = {}
    for evt in prof.events():
        if evt.device_type != torch.autograd.DeviceType.CUDA:
            continue
        name = evt.name
        t = evt.device_time_total if hasattr(evt, "device_time_total") else evt.cuda_time_total
        k = per_kernel.setdefault(name, [0.0, 0])
        k[0] += t / 1e3 / args.steps
        k[1] += 1
    classes = {c: [0.0, 0] for c, _ in KERNEL_CLASSES}
    classes["other ATen / elementwise"] = [0.0, 0]
    for name, (ms, n) in per_kernel.items():
        for c, keys in KERNEL_CLASSES:
            if any(k in name for k in keys):
                break
        else:
            c = "other ATen / elementwise"
        classes[c][0] += ms
        classes[c][1] += n / args.steps
    busy = sum(v[0] for v in classes.values())
    print(f"step: {ev_ms:.2f} ms (CUDA events, unprofiled), kernels {busy:.2f} ms, idle {ev_ms - busy:.2f} ms; "
          f"{n_edges:.0f} edges, {n_nodes:.0f} atoms per step")
    print("| class | ms/step | share of step | launches/step |")
    print("|---|---|---|---|")
    for c, (ms, n) in sorted(classes.items(), key=lambda kv: -kv[1][0]):
        print(f"| {c} | {ms:.2f} | {ms / ev_ms:.3f} | {n:.0f} |")
    print(f"| idle (launch gaps, host sync) | {ev_ms - busy:.2f} | {(ev_ms - busy) / ev_ms:.3f} | |")
    print("\ntop kernels:")
    print("| kernel | ms/step | launches/step |")
    print("|---|---|---|")
    for name, (ms, n) in sorted(per_kernel.items(), key=lambda kv: -kv[1][0])[:30]:
        print(f"| `{name[:110]}` | {ms:.3f} | {n / args.steps:.0f} |")
    print(json.dumps({"breakdown_ms_per_step": ev_ms, "kernel_ms": busy,
                      "classes": {c: round(v[0], 3) for c, v in classes.items()}}), flush=True)


def run_partitioned_inference(args, device, world, rank):
    """Device-scale partitioned inference: a crystalline Si slab with a Hf/O-substituted oxide
    layer, split into spatial slabs, one per rank.  Each rank builds the edges into its own
    atoms on the device (cell-list radius graph, no global edge list), runs the backbone over
    edge chunks (edge stream updated in place, NVLink halo exchange per block) and streams its
    block-sparse Hamiltonian shard (head -> fused CG transform + scatter).  Metric: global
    edges per second.  The e2e arm copies the rank's inputs from pinned memory and its whole
    Hamiltonian shard back to pinned memory every step."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from maloq_b200.data import datasets, structures
    from maloq_b200.data.graph_gpu import radius_graph_device
    from maloq_b200.models.backbone import eSEN_Backbone
    from maloq_b200.models.heads import Fock_Irreps_Head
    from maloq_b200.parallel import dist as pdist
    from maloq_b200.parallel import partition as P
    from maloq_b200.parallel.halo import local_batch
    from maloq_b200.parallel.infer import hamiltonian_shard

    kind, def_atoms, mmax, def_layers, _ = PARTITIONED[args.config]
    n_atoms = args.atoms or def_atoms
    layers = def_layers if args.layers == 6 else args.layers
    t0 = time.time()
    labeler = datasets.labeler_for(kind, device)
    lmax = labeler.layout.lmax
    cutoff = datasets.SPECS[kind]["cutoff"]
    st = structures.si_slab_with_oxide(np.random.default_rng(0), n_atoms)
    part = P.partition("slab", len(st.z), world, pos=st.pos, cell=st.cell)
    owned = np.flatnonzero(part == rank)
    src_g, dst_l, vec, dst_ptr = radius_graph_device(st.pos, cutoff, st.cell, targets=owned, device=device)
    dom, src_local = P.local_domain(part, rank, world, src_g)
    transport = "peer" if world > 1 else "collective"
    batch = local_batch(st.z, st.pos, dom, src_local, dst_l, vec, dst_ptr, labeler.table, device=device,
                        transport=transport)
    del src_g, dst_l, vec, src_local
    host = batch.to("cpu").pin_memory()
    E_local = batch.num_edges
    e_tot = torch.tensor([E_local], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e_tot)
    edges = int(e_tot.item())
    t_graph = time.time() - t0

    torch.manual_seed(1)
    kw = dict(sphere_channels=args.channels, hidden_channels=args.channels, lmax=lmax, mmax=mmax, cutoff=cutoff,
              edge_channels=args.channels, num_layers=layers, num_distance_basis=128, edge_chunk=args.edge_chunk)
    backbone = eSEN_Backbone(labeler.irreps, include_edges=True, **kw).to(device).eval()
    head = Fock_Irreps_Head(None, labeler.irreps, lmax=lmax, sphere_channels=args.channels,
                            ls_list=labeler.layout.ls_list, reduce_node=True, reduce_node_intra=True).to(device).eval()
    buf = [None]

    def step(b):
        with torch.no_grad():
            emb = backbone(b)
            data, ptr = hamiltonian_shard(head, emb, b, labeler, out=buf[0])
            buf[0] = data
            return data, ptr

    host_out = [None]

    def step_e2e(i):
        data, _ = step(host.to(device, non_blocking=True))
        if host_out[0] is None or host_out[0].numel() != data.numel():
            host_out[0] = torch.empty(data.numel(), dtype=data.dtype).pin_memory()
        host_out[0].copy_(data, non_blocking=True)
        return None, None, data[:1].sum()

    ms, e2e_ms, launches, clk, _ = timed_steps(args, device, world, lambda i: step(batch), step_e2e)
    ms_step = ms / args.steps
    if rank == 0:
        out = {
            "metric": "inference edges/s (Si/HfO2 slab partitioned, device-timed, max over ranks)",
            "value": round(edges / (ms_step / 1e3), 1), "unit": "edges/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (diamond Si slab, 10% Hf/O substitution in a 3 nm oxide layer, 0.05 A displacements; "
                    "random-init weights)",
            "config": {"model": f"eSEN lmax={lmax} mmax={mmax} C={args.channels} layers={layers} + Fock head "
                                f"(DZVP-like Si/O 13, Hf 25 orbitals, D={labeler.target_len})",
                       "atoms": len(st.z), "edges": edges, "cutoff_A": cutoff,
                       "edges_per_atom": round(edges / len(st.z), 1), "parallelism": f"graph{world}",
                       "partition": "slab", "halo_transport": transport, "halo_rows_rank0": int(len(dom.halo)),
                       "edges_rank0": int(E_local), "edge_chunk": args.edge_chunk,
                       "output": "block-sparse Hamiltonian shard per rank (fp32 blocks, on device)",
                       "l2": "256 MiB buffer written between timed steps, outside the step events"},
            "e2e": {"value": round(edges / (e2e_ms / args.steps / 1e3), 1), "unit": "edges/s",
                    "h2d_bytes_per_step": int(host.nbytes()),
                    "d2h_bytes_per_step": int(buf[0].numel() * buf[0].element_size() + 4)},
            "gpu_launches": int(launches), "clocks": clk,
            "peak_mem_gb": round(torch.cuda.max_memory_allocated(device) / 2**30, 2),
            "graph_build_s": round(t_graph, 1),
        }
        print(json.dumps(out), flush=True)
    if world > 1:
        pdist.cleanup_process_group()


def run_partitioned(args, device, world, rank):
    """One periodic structure split over the ranks by spatial slabs (graph parallel): each rank
    trains on its owned atoms and the edges into them; halo (ghost) rows are read from the
    owners' memory inside the edge kernels (NVLink peer halo) and their gradients are pushed
    back to the owners; model gradients are summed by the fused all-reduce.  Metric: global
    edges per second.  Every rank builds the same structure from the same seed."""
    import torch
    import torch.distributed as dist

    from maloq_b200.data import datasets
    from maloq_b200.data.targets import Teacher
    from maloq_b200.models.backbone import eSEN_Backbone
    from maloq_b200.models.heads import Fock_Irreps_Head
    from maloq_b200.parallel import dist as pdist
    from maloq_b200.parallel import partition as P
    from maloq_b200.parallel.dp import GradSync
    from maloq_b200.parallel.halo import partition_batch
    from maloq_b200.train import loss as L
    from maloq_b200.train.trainer import SplitTrainer

    kind, def_atoms, mmax, def_layers, _ = PARTITIONED[args.config]
    n_atoms = args.atoms or def_atoms
    layers = def_layers if args.layers == 6 else args.layers
    t0 = time.time()
    labeler = datasets.labeler_for(kind, device)
    lmax = labeler.layout.lmax
    cutoff = datasets.SPECS[kind]["cutoff"]
    sample = datasets.build_samples(kind, 1, seed=0, n_atoms=n_atoms)[0]
    part = P.partition("slab", sample.num_nodes, world, src=sample.src, dst=sample.dst, pos=sample.pos,
                       cell=sample.cell)
    dom = P.decompose(part, sample.src, sample.dst, world)[rank]
    transport = "peer" if world > 1 else "collective"
    batch = partition_batch(sample, dom, labeler.table, device=device, transport=transport)
    kw = dict(sphere_channels=args.channels, hidden_channels=args.channels, lmax=lmax, mmax=mmax, cutoff=cutoff,
              edge_channels=args.channels, num_layers=layers, num_distance_basis=128, edge_chunk=args.edge_chunk)
    teacher = Teacher(kw, labeler, device=device)
    with torch.no_grad():
        no, eo = teacher.head(teacher.backbone(batch), batch)
    batch.node_y, batch.y = no.detach().clone(), eo.detach().clone()
    del teacher, no, eo
    torch.cuda.empty_cache()
    host = batch.to("cpu").pin_memory()
    t_data = time.time() - t0

    torch.manual_seed(1)
    backbone = eSEN_Backbone(labeler.irreps, include_edges=True, **kw).to(device)
    head = Fock_Irreps_Head(None, labeler.irreps, lmax=lmax, sphere_channels=args.channels,
                            ls_list=labeler.layout.ls_list, reduce_node=True, reduce_node_intra=True).to(device)
    params = list(backbone.parameters()) + list(head.parameters())
    opt = torch.optim.Adam(params, lr=1e-4, fused=True)
    sync = GradSync(params, mode=args.grad_sync or "fused") if world > 1 else None
    trainer = SplitTrainer(backbone, head, labeler.irreps, mask_table=torch.as_tensor(labeler.table.mask),
                           grad_sync=sync)
    loss_fn = L.rmse_mse_padded_loss
    ms, e2e_ms, launches, clk, loss_vals = timed_steps(
        args, device, world, lambda i: trainer.train_step(batch, loss_fn, opt),
        lambda i: trainer.train_step(host.to(device, non_blocking=True), loss_fn, opt))
    ms_step = ms / args.steps
    edges = sample.num_edges
    h2d = host.nbytes()
    if rank == 0:
        out = {
            "metric": "train edges/s (Si/O partitioned, device-timed, max over ranks)",
            "value": round(edges / (ms_step / 1e3), 1), "unit": "edges/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random amorphous Si/O supercell, frozen random-init teacher targets; random-init "
                    "weights)",
            "config": {"model": f"eSEN lmax={lmax} mmax={mmax} C={args.channels} layers={layers} + Fock head "
                                f"(DZVP-like, D={labeler.target_len})",
                       "atoms": sample.num_nodes, "edges": edges, "cutoff_A": cutoff,
                       "edges_per_atom": round(edges / sample.num_nodes, 1), "parallelism": f"graph{world}",
                       "partition": "slab", "halo_transport": transport,
                       "halo_rows_rank0": int(len(dom.halo)), "edges_rank0": int(len(dom.edges)),
                       "l2": "256 MiB buffer written between timed steps, outside the step events",
                       "edge_chunk": args.edge_chunk, "edge_stream": "bf16 storage, fp32 compute"},
            "e2e": {"value": round(edges / (e2e_ms / args.steps / 1e3), 1), "unit": "edges/s",
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": 4},
            "gpu_launches": int(launches), "clocks": clk, "final_loss": loss_vals[-1],
            "peak_mem_gb": round(torch.cuda.max_memory_allocated(device) / 2**30, 2),
            "setup_s": round(t_data, 1),
        }
        print(json.dumps(out), flush=True)
    if world > 1:
        pdist.cleanup_process_group()


def run_cpu_plumbing(args):
    """The CPU configuration (no GPU): 8 random molecules of 3-9 atoms from {H,C,N,O}, 5 A graph,
    split-valence basis, lmax 4, mmax 2, 64 channels, 4 layers, 32 Gaussians, MSE loss, 100 Adam
    steps, fixed seeds.  Reports the wall time of the 100 steps, the loss drop and the fp32
    equivariance error of the node and edge outputs under a random rotation (max |D y(x) -
    y(R x)| / max |y|)."""
    import numpy as np
    import torch

    from maloq_b200.core import sph
    from maloq_b200.data import datasets, structures
    from maloq_b200.data.batch import collate, make_sample
    from maloq_b200.models.backbone import eSEN_Backbone
    from maloq_b200.models.heads import Fock_Irreps_Head
    from maloq_b200.train import loss as L
    from maloq_b200.train.trainer import SplitTrainer

    torch.manual_seed(0)
    steps = 100
    kw = dict(sphere_channels=64, hidden_channels=64, lmax=4, mmax=2, cutoff=5.0, edge_channels=64, num_layers=4,
              num_distance_basis=32)
    labeler = datasets.labeler_for("small", "cpu")
    samples, _ = datasets.build_dataset("small", 8, kw, seed=0, device="cpu", labeler=labeler)
    batch = collate(samples, labeler.table)
    torch.manual_seed(1)
    bb = eSEN_Backbone(labeler.irreps, include_edges=True, **kw)
    hd = Fock_Irreps_Head(None, labeler.irreps, lmax=4, sphere_channels=64, ls_list=labeler.layout.ls_list,
                          reduce_node=True, reduce_node_intra=True)
    opt = torch.optim.Adam(list(bb.parameters()) + list(hd.parameters()), lr=1e-3)
    tr = SplitTrainer(bb, hd, labeler.irreps, mask_table=torch.as_tensor(labeler.table.mask))
    t0 = time.time()
    losses = [float(tr.train_step(batch, L.mse_padded_loss, opt)[2]) for _ in range(steps)]
    wall = time.time() - t0
    # equivariance: rotate the input structures (x, y, z); the model frame is (y, z, x)
    rng = np.random.default_rng(9)
    q = rng.normal(size=4)
    q /= np.linalg.norm(q)
    a, b_, c, d = q
    R = np.array([[a * a + b_ * b_ - c * c - d * d, 2 * (b_ * c - a * d), 2 * (b_ * d + a * c)],
                  [2 * (b_ * c + a * d), a * a - b_ * b_ + c * c - d * d, 2 * (c * d - a * b_)],
                  [2 * (b_ * d - a * c), 2 * (c * d + a * b_), a * a - b_ * b_ - c * c + d * d]])
    P = np.array([[0.0, 1.0, 0.0], [0.0, 0.0, 1.0], [1.0, 0.0, 0.0]])
    rot = [make_sample(structures.Structure(s.z, s.pos @ R.T), 5.0) for s in samples]
    b1 = collate(rot, labeler.table)
    with torch.no_grad():
        n0, e0 = hd(bb(batch), batch)
        n1, e1 = hd(bb(b1), b1)
    Dl = torch.block_diag(*[torch.tensor(sph.wigner_D_from_matrix(it.l, P @ R @ P.T), dtype=torch.float32)
                            for it in labeler.irreps])
    scale = max(n0.abs().max().item(), e0.abs().max().item(), 1e-12)
    eq = max((n0[0] @ Dl.T - n1[0]).abs().max().item(), (e0[0] @ Dl.T - e1[0]).abs().max().item()) / scale
    print(json.dumps({
        "metric": "CPU plumbing: wall time of 100 Adam steps", "value": round(wall, 3), "unit": "s", "n_gpus": 0,
        "steps": steps, "warmup": 0, "higher_is_better": False, "dtype": "fp32", "data": "synthetic",
        "config": {"model": "eSEN lmax=4 mmax=2 C=64 layers=4, 32 Gaussians + Fock head", "global_batch": 8,
                   "molecules": "3-9 atoms {H,C,N,O}", "loss": "mse"},
        "loss_first": losses[0], "loss_last": losses[-1], "equivariance_rel_err_fp32": eq}), flush=True)


def main():
    args = parse()
    if args.config == "cpu":
        return run_cpu_plumbing(args)
    if args.impl == "reference":
        out = reference_arm(args)
        if int(os.environ.get("RANK", "0")) == 0 and out is not None:
            print(json.dumps(out))
        return
    sys.path.insert(0, HERE)
    import torch
    import torch.distributed as dist

    from maloq_b200 import ops
    from maloq_b200.data import batch as B
    from maloq_b200.data import datasets
    from maloq_b200.models.backbone import eSEN_Backbone
    from maloq_b200.models.heads import Fock_Irreps_Head
    from maloq_b200.parallel import dist as pdist
    from maloq_b200.parallel.dp import GradSync
    from maloq_b200.train import loss as L
    from maloq_b200.train.trainer import SplitTrainer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        device = pdist.setup_env(backend="nccl")
    else:
        device = torch.device("cuda", 0)
        torch.cuda.set_device(device)
    rank = pdist.rank()
    if args.impl == "torch":
        ops.use_torch_ops(True)
    torch.manual_seed(0)
    if args.config in PARTITIONED:
        if PARTITIONED[args.config][4] == "infer":
            return run_partitioned_inference(args, device, world, rank)
        return run_partitioned(args, device, world, rank)

    kind, mmax, def_layers, per_batch, atom_cap = CONFIGS[args.config]
    if args.config != "druglike" and args.layers == 6:
        args.layers = def_layers
    labeler = datasets.labeler_for(kind, device)
    lmax = labeler.layout.lmax
    kw = dict(sphere_channels=args.channels, hidden_channels=args.channels, lmax=lmax, mmax=mmax, cutoff=6.0,
              edge_channels=args.channels, num_layers=args.layers, num_distance_basis=128)
    t0 = time.time()
    if per_batch is not None:
        n_mol = args.batch * args.n_batches
    else:  # atom-capped batches: enough molecules (mean 80 atoms) for n_batches full batches
        n_mol = args.n_batches * atom_cap // 80
    samples, _ = datasets.build_dataset(kind, n_mol, kw, seed=1000 + rank, device=device, labeler=labeler)
    groups = B.batches_by_count(samples, args.batch) if per_batch is not None else \
        B.batches_by_atoms(samples, atom_cap)[:args.n_batches]
    host_batches = [B.collate(g, labeler.table).pin_memory() for g in groups]
    graphs_per_batch = [len(g) for g in groups]
    dev_batches = [b.to(device) for b in host_batches]
    n_edges = sum(b.num_edges for b in host_batches) / len(host_batches)
    n_nodes = sum(b.num_nodes for b in host_batches) / len(host_batches)
    t_data = time.time() - t0

    torch.manual_seed(1)
    # the large config's 8 layers of edge activations (~260k edges, lmax 6) exceed device memory
    # without recompute: each block is recomputed in backward
    backbone = eSEN_Backbone(labeler.irreps, include_edges=True, activation_checkpointing=args.config == "large",
                             **kw).to(device)
    head = Fock_Irreps_Head(None, labeler.irreps, lmax=lmax, sphere_channels=args.channels,
                            ls_list=labeler.layout.ls_list, reduce_node=True, reduce_node_intra=True).to(device)
    params = list(backbone.parameters()) + list(head.parameters())
    opt = torch.optim.Adam(params, lr=1e-4, fused=True)
    sync = None
    if world > 1:
        mode = args.grad_sync or ("nccl" if args.impl == "torch" else "fused")
        sync = GradSync(params, mode=mode)
    trainer = SplitTrainer(backbone, head, labeler.irreps, mask_table=torch.as_tensor(labeler.table.mask),
                           grad_sync=sync)
    loss_fn = L.rmse_mse_padded_loss
    if args.breakdown:
        return step_breakdown(args, lambda i: trainer.train_step(dev_batches[i % len(dev_batches)], loss_fn, opt),
                              n_edges, n_nodes)
    ms, e2e_ms, launches, clk, loss_vals = timed_steps(
        args, device, world, lambda i: trainer.train_step(dev_batches[i % len(dev_batches)], loss_fn, opt),
        lambda i: trainer.train_step(host_batches[i % len(host_batches)].to(device, non_blocking=True), loss_fn,
                                     opt))
    # equivariance of the timed model on the product path (bf16 GEMM operands), outside the timing
    import numpy as np

    from maloq_b200.data import structures as S_
    from maloq_b200.eval.equivariance import model_equivariance_error, random_rotation

    rng_eq = np.random.default_rng(7)
    mols_eq = [S_.random_druglike_molecule(rng_eq, 30, 50) for _ in range(4)] if kind == "druglike" else []
    eq_err = (model_equivariance_error(backbone, head, mols_eq, labeler, 6.0, random_rotation(rng_eq), device)
              if mols_eq and args.impl == "native" else None)
    nbytes = [sum(v.numel() * v.element_size() for v in hb.tensors().values()) for hb in host_batches]
    h2d = sum(nbytes[i % len(nbytes)] for i in range(args.steps)) / args.steps

    ms_step = ms / args.steps
    # graphs per step on this rank, averaged over the timed steps (batches cycle); weak scaling
    graphs = world * sum(graphs_per_batch[i % len(graphs_per_batch)] for i in range(args.steps)) / args.steps
    value = graphs / (ms_step / 1e3)
    e2e_value = graphs / (e2e_ms / args.steps / 1e3)
    if rank == 0:
        out = {
            "metric": METRIC if args.config == "druglike" else
            "train graphs/s (large molecules DP, device-timed, max over ranks)", "value": round(value, 2), "unit": "graphs/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None if BASELINE_VALUE is None else value / BASELINE_VALUE,
            "dtype": "bf16" if args.impl == "native" else "fp32",
            "data": f"synthetic (random {kind} molecules, frozen random-init teacher targets; random-init weights)",
            "config": {"model": f"eSEN lmax={lmax} mmax={mmax} C={args.channels} layers={args.layers} + Fock head "
                                f"({labeler_name(kind)}, D={labeler.target_len})",
                       "global_batch": round(graphs, 2), "atoms_cap_per_gpu": atom_cap, "seq_len": None, "parallelism": f"dp{world}",
                       "edges_per_gpu_step": round(n_edges), "atoms_per_gpu_step": round(n_nodes),
                       "l2": "256 MiB buffer written between timed steps, outside the step events",
                       "impl": args.impl, "grad_sync": None if sync is None else sync.mode,
                       "allreduce_transport": (sync._fused.transport if sync is not None and sync._fused is not None
                                               else ("nccl" if sync is not None else None))},
            "e2e": {"value": round(e2e_value, 2), "unit": "graphs/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": 4},
            "gpu_launches": int(launches),
            "clocks": clk,
            "final_loss": loss_vals[-1],
            "equivariance_rel_err_bf16": None if eq_err is None else float(f"{eq_err:.3g}"),
            "peak_mem_gb": round(torch.cuda.max_memory_allocated(device) / 2**30, 2),
            "activation_checkpointing": backbone.activation_checkpointing,
            "setup_s": round(t_data, 1),
        }
        print(json.dumps(out), flush=True)
    if world > 1:
        pdist.cleanup_process_group()


if __name__ == "__main__":
    main()
