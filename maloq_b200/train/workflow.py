"""TrainingWorkflow: config -> data -> model -> train / eval / infer (reference
``train_utils/training_workflow.py``).

Same public API as the reference: ``TrainingWorkflow(config).run()`` with the reference's
config keys (plus ``mmax``, ``grad_sync``, ``num_structures``).  Datasets:

* ``synthetic_small`` / ``synthetic_druglike`` / ``synthetic_large`` / ``synthetic_sio2`` -
  generated structures with teacher targets (:mod:`maloq_b200.data.datasets`);
* ``nablaDFT`` - the nablaDFT SQLite Hamiltonian database (:mod:`maloq_b200.data.readers`).

``rcut_orbitals`` is a per-atom radius, so graphs connect pairs closer than
``2 * rcut_orbitals`` (reference ``fock_targets_batched.py:208``); ``rcut_gaussian`` is the
Gaussian-smearing range.
"""

from __future__ import annotations

import json
import os
import random

import numpy as np
import torch

from ..data import batch as B
from ..data import datasets
from ..models.backbone import eSEN_Backbone
from ..models.heads import Fock_Irreps_Head, HELM_Energy_Head, HELM_Force_Head
from ..parallel import dist as pdist
from . import checkpoint as ckpt
from . import loss as L
from .trainer import SplitTrainer


class TrainingWorkflow:
    DEFAULTS = {
        "run_name": "run", "output_folder": "outputs", "open_shell": False,
        "device": "cuda" if torch.cuda.is_available() else "cpu", "wigner_backend": "cuda",
        "distribute_graphs": False, "partition_type": None, "tiling_dims": None, "lr_init": 1e-4,
        "optimizer_type": "adam", "compute_total_energy": False,
        "dist_backend": "nccl" if torch.cuda.is_available() else "gloo",
        "dtype": torch.float32, "train_or_eval": "train", "train_backbone": True, "train_head": True,
        "restart_backbone": False, "restart_head": False, "restart_optimizer": False,
        "backbone_checkpoint": "backbone.pt", "head_checkpoint": "head.pt", "reduce_edge": False,
        "reduce_node": True, "reduce_node_intra": True, "loss_target": "fock_matrix", "num_epochs": 1,
        "batch_size": 1, "scheduler_type": "cosine", "eta_min": 1e-8, "patience": 100, "threshold": 1e-8,
        "save_frequency": 10, "num_distance_basis": 128, "num_mp_layers": 3, "l_embedding_dim": 128,
        "rcut_orbitals": 3.0, "rcut_gaussian": 6.0, "gaussian_width": 1.0,
        "train_loss_fxn": L.rmse_mse_padded_loss, "test_loss_fxn": L.l1_unpadded_loss,
        "dataset_name": "synthetic_small", "num_structures": 16, "num_train": 0, "num_val": 0,
        "grad_sync": None, "seed": 42,
    }

    def __init__(self, config):
        self.config = self.DEFAULTS | dict(config)
        for k in ("train_loss_fxn", "test_loss_fxn"):
            self.config[k] = L.get_loss(self.config[k])
        self.setup_environment()
        self.check_input_config()

    def setup_environment(self):
        seed = self.config["seed"]
        torch.manual_seed(seed)
        np.random.seed(seed)
        random.seed(seed)
        torch.set_default_dtype(self.config["dtype"] if self.config["dtype"] != torch.bfloat16 else torch.float32)
        self.rank, self.world_size, _ = pdist.env_rank_world()
        if self.config["device"] == "cpu":
            self.config["dist_backend"] = "gloo"
        if self.world_size > 1 or self.config["distribute_graphs"]:
            self.device = pdist.setup_env(backend=self.config["dist_backend"])
            if self.config["device"] == "cpu":
                self.device = torch.device("cpu")
        else:
            self.device = torch.device(self.config["device"])
            if self.device.type == "cuda":
                torch.cuda.set_device(self.device)
        if self.rank == 0:
            os.makedirs(self.config["output_folder"], exist_ok=True)

    def check_input_config(self):
        c = self.config
        c["include_edges"] = "matrix" in c["loss_target"]
        if c.get("hidden_dim") is None:
            c["hidden_dim"] = c["l_embedding_dim"]
        c.setdefault("message_type", "source-target")
        c.setdefault("activation_checkpointing", False)
        # device error word read every N steps (multi-GPU runs default to 50); 0: per epoch only
        c.setdefault("device_status_every", 50 if self.world_size > 1 else 0)
        c.setdefault("basis_transform_backend", "cuda")
        if c["distribute_graphs"] and c["partition_type"] is None:
            c["partition_type"] = "slab"
        if c["reduce_edge"] and c["distribute_graphs"]:
            raise ValueError("reduce_edge and distribute_graphs cannot both be True")
        if c["distribute_graphs"] and "matrix" not in c["loss_target"]:
            raise ValueError("distributed graph training needs a matrix-valued loss target")
        for name, key in (("backbone", "restart_backbone"), ("head", "restart_head")):
            if c[key]:
                path = os.path.join(c["output_folder"], c[f"{name}_checkpoint"])
                if not os.path.exists(path):
                    raise FileNotFoundError(f"{name} checkpoint not found at {path}")
                try:
                    torch.load(path, map_location="cpu", weights_only=False)
                except Exception as e:  # noqa: BLE001 - report which file is corrupt
                    raise ValueError(f"Error loading {name} checkpoint from {path}: {e}") from e
        if self.rank == 0 and c["train_or_eval"] == "train":
            path = os.path.join(c["output_folder"], f"config_{c['run_name']}.json")
            with open(path, "w") as f:
                json.dump({k: (v.__name__ if hasattr(v, "__name__") else str(v)) for k, v in c.items()}, f, indent=4)

    # ------------------------------------------------------------------ data
    def model_kwargs(self, lmax):
        c = self.config
        mmax = c.get("mmax") or lmax
        return dict(sphere_channels=c["l_embedding_dim"], hidden_channels=c["hidden_dim"], lmax=lmax,
                    mmax=min(mmax, lmax), cutoff=c["rcut_gaussian"], edge_channels=c["l_embedding_dim"],
                    num_layers=c["num_mp_layers"], num_distance_basis=c["num_distance_basis"],
                    gaussian_width=c["gaussian_width"], message_type=c["message_type"], open_shell=c["open_shell"],
                    activation_checkpointing=c["activation_checkpointing"], edge_chunk=c.get("edge_chunk"),
                    norm_type=c.get("norm_type", "rms_norm_sh"))

    def prepare_partitioned(self):
        """One structure split over the ranks (graph parallel): rank 0 generates it (or every
        rank reads the same CP2K structure, ``dataset_name: cp2k``), every rank builds the same
        partition, keeps its domain, and takes its nodes'/edges' targets (read ones, or the
        partitioned teacher's for synthetic structures; reference
        ``fock_targets_batched.py:231-333``)."""
        import torch.distributed as dist

        from ..data.targets import Teacher
        from ..parallel import partition as P
        from ..parallel.halo import partition_batch

        c = self.config
        name = c["dataset_name"]
        kind = name[len("synthetic_"):] if name.startswith("synthetic_") else name
        if name != "cp2k" and kind not in ("sio2", "slab"):
            return self.prepare_partitioned_molecules()
        if name == "cp2k":
            samples, labeler = self._load_cp2k_folder(dict(c, num_structures=c.get("structure_index", 0) + 1))
            sample = samples[c.get("structure_index", 0)]
        else:
            labeler = datasets.labeler_for(kind, self.device)
            obj = [None]
            if self.rank == 0:
                obj[0] = datasets.build_samples(kind, 1, seed=c["seed"], cutoff=2 * c["rcut_orbitals"],
                                                n_atoms=c.get("num_atoms", 20000))[0]
            if dist.is_initialized():
                dist.broadcast_object_list(obj, src=0)
            sample = obj[0]
        world = self.world_size if dist.is_initialized() else 1
        part = P.partition(c["partition_type"], sample.num_nodes, world, src=sample.src, dst=sample.dst,
                           pos=sample.pos, cell=sample.cell)
        dom = P.decompose(part, sample.src, sample.dst, world)[self.rank if dist.is_initialized() else 0]
        transport = c.get("halo_transport") or ("peer" if self.device.type == "cuda" and world > 1 else "collective")
        batch = partition_batch(sample, dom, labeler.table, device=self.device, transport=transport)
        if c["train_or_eval"] != "infer" and sample.node_y is None:
            teacher = Teacher(self.model_kwargs(labeler.layout.lmax), labeler, device=self.device)
            with torch.no_grad():
                no, eo = teacher.head(teacher.backbone(batch), batch)
            batch.node_y, batch.y = no.detach().clone(), eo.detach().clone()
        self.labeler = labeler
        self.val_samples = []
        self.partition_sample = sample
        return [batch], [batch], labeler

    def prepare_partitioned_molecules(self):
        """``distribute_graphs`` on a molecule dataset: batches of molecules become single graphs
        (disjoint unions, "supergraphs") split over all ranks; every rank keeps its domain of
        every supergraph, so all ranks hold the same number of batches in the same order.
        Each rank first takes its share of the molecules.  Two ways to form the supergraphs
        (reference ``dataset_utils/get_loader.py:237-413``):

        * training (``all_ranks_contribute``): supergraph i is the union of molecules
          [i·batch_size, (i+1)·batch_size) of every rank's share, in rank order (all-gathered);
        * evaluation (``one_rank_contributes``): the ranks take turns as the source,
          broadcasting their share ``batch_size`` molecules at a time.
        """
        import torch.distributed as dist

        from ..parallel import partition as P
        from ..parallel.halo import partition_batch

        c = self.config
        samples, labeler = self._load_global_samples(c)
        n_val = c["num_val"] or max(1, len(samples) // 8)
        n_train = c["num_train"] or (len(samples) - n_val)
        train, val = samples[:n_train], samples[n_train:n_train + n_val]
        if c.get("scale_and_shift"):
            self.scale_shift, self.energy_refs = None, None
            self._apply_scale_shift(train, samples, labeler, c["dataset_name"])
        on = dist.is_initialized() and self.world_size > 1
        world, rank = (self.world_size, self.rank) if on else (1, 0)
        bs = c["batch_size"]
        mode = "one_rank_contributes" if c["train_or_eval"] == "eval" else "all_ranks_contribute"
        # GPUs: the halos of molecule batches are small; the collective transport needs no
        # per-batch symmetric-memory buffers
        transport = c.get("halo_transport") or "collective"

        def split(g):
            part = P.partition(c["partition_type"], g.num_nodes, world, src=g.src, dst=g.dst, pos=g.pos)
            dom = P.decompose(part, g.src, g.dst, world)[rank]
            return partition_batch(g, dom, labeler.table, device=self.device, transport=transport)

        def batches(pool):
            mine = [pool[i] for i in pdist.split_indices(len(pool), rank, world, drop_remainder=False)]
            counts = [len(mine)]
            if on:
                counts = [None] * world
                dist.all_gather_object(counts, len(mine))
            groups = []
            if mode == "all_ranks_contribute":
                for i in range(0, max(counts), bs):
                    parts = [mine[i:i + bs]]
                    if on:
                        parts = [None] * world
                        dist.all_gather_object(parts, mine[i:i + bs])
                    groups.append([m for p in parts for m in p])
            else:
                for src_rank in range(world):
                    for i in range(0, counts[src_rank], bs):
                        obj = [mine[i:i + bs] if src_rank == rank else None]
                        if on:
                            dist.broadcast_object_list(obj, src=src_rank)
                        groups.append(obj[0])
            return [split(B.merge_samples(g)) for g in groups], groups

        self.labeler = labeler
        self.val_samples = []
        self.supergraph_mode = mode
        tr, _ = batches(train)
        va, self.val_groups = batches(val)
        return tr, va, labeler

    def _load_global_samples(self, c):
        """All molecules of a dataset that every rank reads whole (synthetic, nablaDFT, QM7, one
        ASE database file)."""
        name = c["dataset_name"]
        if name.startswith("synthetic_"):
            kind = name[len("synthetic_"):]
            labeler = datasets.labeler_for(kind, self.device)
            return datasets.build_dataset(kind, c["num_structures"], self.model_kwargs(labeler.layout.lmax),
                                          seed=c["seed"], device=self.device, cutoff=2 * c["rcut_orbitals"],
                                          labeler=labeler, target=c["loss_target"])
        if name == "nablaDFT":
            from ..data.readers import load_nabladft

            return load_nabladft(c["dbpath"], c, self.device)
        if name == "QM7":
            from ..data.readers import load_qm7

            return load_qm7(c["dbpath"], c, self.device)
        if str(c.get("dbpath", "")).endswith(".db"):
            from ..data.readers import load_ase_entries

            return load_ase_entries([{"db_file": c["dbpath"], "start_idx": 0, "end_idx": None}], c, self.device,
                                    basis=c.get("basis_name", "def2_tzvpd"))
        raise ValueError(f"distribute_graphs: dataset {name!r} is not a molecule dataset read whole by every rank")

    def _load_cp2k_folder(self, c):
        """``dbpath``: a folder of structure directories, each with ``structure.xyz`` and
        ``hamiltonian.csr`` (CP2K dump), optionally ``overlap.csr`` + ``cp2k.out`` for the
        Fermi-level shift.  Basis: ``basis_name`` (default the DZVP-like Si/O/Hf basis).
        ``tiling_dims`` replicates each cell into a supercell with the cell's targets."""
        from ..data.readers import load_cp2k

        root = c["dbpath"]
        dirs = sorted(d for d in os.listdir(root) if os.path.isfile(os.path.join(root, d, "structure.xyz")))
        samples, labeler = [], None
        for d in dirs[: c.get("num_structures") or len(dirs)]:
            p = os.path.join(root, d)
            s_path, o_path = os.path.join(p, "overlap.csr"), os.path.join(p, "cp2k.out")
            s, labeler = load_cp2k(os.path.join(p, "structure.xyz"), os.path.join(p, "hamiltonian.csr"), c,
                                   basis_name=c.get("basis_name", "dzvp_like"),
                                   s_path=s_path if os.path.exists(s_path) else None,
                                   out_path=o_path if os.path.exists(o_path) else None, device=self.device)
            samples.append(s)
        if not samples:
            raise ValueError(f"no CP2K structure directories under {root}")
        return samples, labeler

    def _apply_scale_shift(self, train, samples, labeler, name):
        """``scale_and_shift``: Fock targets get the per-element mean of their l=0 on-site
        entries subtracted (tables ``element_scale_shifts_{dataset}.pt`` in the output folder,
        loaded if present, else computed from the training set and saved); energy targets get
        per-element linear references (least squares of E on element counts, saved as
        ``lin_ref_coeffs_{dataset}.npz`` with ``coeff[Z]``) subtracted.  Reference
        ``training_workflow.py:150-228``."""
        import numpy as np

        from ..data.targets import ScaleShift

        c = self.config
        os.makedirs(c["output_folder"], exist_ok=True)
        if c["loss_target"] in ("fock_matrix", "density_matrix"):
            from ..data.tools import scale_shift_table

            path = os.path.join(c["output_folder"], f"element_scale_shifts_{name}.pt")
            spins = int(train[0].node_y.shape[0]) if train else 1
            suffixes = [""] if spins == 1 else ["_alpha", "_beta"]
            if os.path.exists(path):
                d = torch.load(path, weights_only=False)
            else:
                d = scale_shift_table(train, labeler)
                if self.rank == 0:
                    torch.save(d, path)
            # one table per spin channel (open shell: keys suffixed _alpha / _beta)
            per_spin = [ScaleShift(labeler, means={int(z): torch.as_tensor(v) for z, v in
                                                   d["element_scalar_means" + sf].items()}) for sf in suffixes]
            for s in samples:
                s.node_y = torch.stack([ss.shift(s.node_y[k], s.z) for k, ss in enumerate(per_spin)])
            ss = per_spin[0]
            self.scale_shift = ss
            self.scale_shifts = per_spin
        elif c["loss_target"] == "energies":
            path = os.path.join(c["output_folder"], f"lin_ref_coeffs_{name}.npz")
            if os.path.exists(path):
                coeff = np.load(path)["coeff"]
            else:
                zmax = max(int(s.z.max()) for s in samples)
                A = np.stack([np.bincount(s.z, minlength=zmax + 1) for s in train]).astype(np.float64)
                coeff = np.linalg.lstsq(A, np.array([s.energy for s in train]), rcond=None)[0]
                if self.rank == 0:
                    np.savez(path, coeff=coeff)
            for s in samples:
                s.energy = s.energy - float(np.bincount(s.z, minlength=len(coeff))[: len(coeff)] @ coeff)
            self.energy_refs = coeff

    def prepare_data(self):
        c = self.config
        if c["distribute_graphs"]:
            return self.prepare_partitioned()
        name = c["dataset_name"]
        if name.startswith("synthetic_") or name in ("nablaDFT", "QM7"):
            samples, labeler = self._load_global_samples(c)
        elif name == "cp2k":
            samples, labeler = self._load_cp2k_folder(c)
        elif name == "omol_csh_58k":
            from ..data.readers import load_omol_csh

            n_tr, n_va = c["num_train"], c["num_val"]
            if not n_tr:
                raise ValueError("omol_csh_58k needs num_train (and num_val) to pick rows of the manifest")
            tr = pdist.split_indices(n_tr, self.rank, self.world_size, drop_remainder=False)
            va = [n_tr + i for i in pdist.split_indices(n_va, self.rank, self.world_size, drop_remainder=False)]
            local, labeler = load_omol_csh(c["dbpath"], c, self.device, indices=list(tr) + va)
            return self._finish_data(local[:len(tr)], local[len(tr):], local, labeler, name, rank_local=True)
        elif os.path.isdir(str(c.get("dbpath", ""))) or str(c.get("dbpath", "")).endswith(".db"):
            # ASE databases (e.g. OMol folders of .db files): each rank reads only its segments
            from ..data.asedb import distribute_data
            from ..data.readers import load_ase_entries

            src = c["dbpath"]
            if os.path.isdir(str(src)):
                tr_e, va_e = distribute_data(src, self.world_size, self.rank, c["num_train"], c["num_val"])
                train, labeler = load_ase_entries(tr_e, c, self.device, basis=c.get("basis_name", "def2_tzvpd"))
                val = load_ase_entries(va_e, c, self.device, basis=c.get("basis_name", "def2_tzvpd"))[0] \
                    if va_e else []
                return self._finish_data(train, val, train + val, labeler, name, rank_local=True)
            samples, labeler = load_ase_entries([{"db_file": src, "start_idx": 0, "end_idx": None}], c,
                                                self.device, basis=c.get("basis_name", "def2_tzvpd"))
        else:
            raise ValueError(f"Unknown dataset name: {name}")
        n_val = c["num_val"] or max(1, len(samples) // 8)
        n_train = c["num_train"] or (len(samples) - n_val)
        train, val = samples[:n_train], samples[n_train:n_train + n_val]
        if name == "nablaDFT" and c.get("dbpath_val"):  # a separate validation database
            from ..data.readers import load_nabladft

            val, _ = load_nabladft(c["dbpath_val"], c, self.device)
            samples = train + val
        return self._finish_data(train, val, samples, labeler, name)

    def _finish_data(self, train, val, samples, labeler, name, rank_local=False):
        """Scale/shift, the data-parallel split (unless each rank read only its own rows) and
        batching."""
        c = self.config
        self.scale_shift, self.energy_refs = None, None
        if c.get("scale_and_shift"):
            self._apply_scale_shift(train, samples, labeler, name)
        if self.world_size > 1 and not c["distribute_graphs"] and not rank_local:
            train = [train[i] for i in pdist.split_indices(len(train), self.rank, self.world_size)]
            val = [val[i] for i in pdist.split_indices(len(val), self.rank, self.world_size, drop_remainder=False)] or val[:1]
        bs = c["batch_size"]
        mk = lambda xs: [B.collate(g, labeler.table).pin_memory() if self.device.type == "cuda"
                         else B.collate(g, labeler.table) for g in B.batches_by_count(xs, bs, drop_last=False)]
        self.labeler = labeler
        self.val_samples = val
        return mk(train), mk(val), labeler

    # ------------------------------------------------------------------ model
    def build_model(self, labeler):
        c = self.config
        irreps = labeler.irreps
        lmax = irreps.lmax
        backbone = eSEN_Backbone(irreps, include_edges=c["include_edges"], **self.model_kwargs(lmax)).to(self.device)
        if c["loss_target"] in ("fock_matrix", "density_matrix"):
            head = Fock_Irreps_Head(None, irreps, lmax=lmax, sphere_channels=c["l_embedding_dim"],
                                    reduce_edge=c["reduce_edge"], open_shell=c["open_shell"],
                                    ls_list=labeler.layout.ls_list, reduce_node=c["reduce_node"],
                                    reduce_node_intra=c["reduce_node_intra"])
        elif c["loss_target"] == "forces":
            head = HELM_Force_Head(backbone)
        else:
            head = HELM_Energy_Head(backbone)
        head = head.to(self.device)
        params = []
        for m, flag in ((backbone, c["train_backbone"]), (head, c["train_head"])):
            if flag:
                params += list(m.parameters())
            else:
                for p in m.parameters():
                    p.requires_grad_(False)
        if c["optimizer_type"] == "adamw":
            opt = torch.optim.AdamW(params, lr=c["lr_init"], weight_decay=c.get("weight_decay", 0.0))
        elif c["optimizer_type"] == "muon":
            opt = L.HybridMuon(params, muon_lr=c.get("muon_lr", 0.02), adamw_lr=c["lr_init"],
                               weight_decay=c.get("weight_decay", 0.0))
        else:
            opt = torch.optim.Adam(params, lr=c["lr_init"], **({"fused": True} if self.device.type == "cuda" else {}))
        folder = c["output_folder"]
        if c["restart_backbone"]:
            ckpt.load_model(backbone, os.path.join(folder, c["backbone_checkpoint"]), self.device)
        if c["restart_head"]:
            ckpt.load_model(head, os.path.join(folder, c["head_checkpoint"]), self.device,
                            opt if c["restart_optimizer"] else None)
        return backbone, head, opt

    def get_scheduler(self, optimizer, n_batches):
        c = self.config
        if c["scheduler_type"] == "plateau":
            return torch.optim.lr_scheduler.ReduceLROnPlateau(optimizer, mode="min", factor=0.5,
                                                              patience=c["patience"], threshold=c["threshold"])
        return torch.optim.lr_scheduler.CosineAnnealingLR(optimizer, T_max=max(1, c["num_epochs"] * n_batches),
                                                          eta_min=c["eta_min"])

    def grad_sync(self, backbone, head):
        if self.world_size <= 1:
            return None
        from ..parallel.dp import GradSync

        mode = self.config["grad_sync"] or ("fused" if self.device.type == "cuda" else "nccl")
        params = [p for p in list(backbone.parameters()) + list(head.parameters()) if p.requires_grad]
        return GradSync(params, mode=mode)

    # ------------------------------------------------------------------ run
    def run(self):
        try:
            c = self.config
            train, val, labeler = self.prepare_data()
            backbone, head, opt = self.build_model(labeler)
            sched = self.get_scheduler(opt, len(train))
            mask_table = torch.as_tensor(labeler.table.mask)
            trainer = SplitTrainer(backbone, head, labeler.irreps, save_frequency=c["save_frequency"],
                                   run_name=c["run_name"], mask_table=mask_table,
                                   grad_sync=self.grad_sync(backbone, head),
                                   status_every=c["device_status_every"],
                                   uncoupled_loss_transform=labeler.transform if c.get("compute_uncoupled_loss")
                                   else None)
            if c["train_or_eval"] == "train":
                if c["restart_backbone"] or c["restart_head"]:
                    st = ckpt.load_resume(c["output_folder"], sched)
                    if st is not None:
                        trainer.start_epoch = st["epoch"] + 1
                        trainer.history = st["history"]
                return trainer.train(c["num_epochs"], c["train_loss_fxn"], opt, sched, self.device, train,
                                     val_loader=val, output_folder=c["output_folder"],
                                     step_every_epoch=c["step_every_epoch"] if "step_every_epoch" in c else False,
                                     log_every=c.get("log_every", 1))
            if c["train_or_eval"] == "eval" and getattr(self, "val_groups", None) is not None:
                return trainer.evaluate_partitioned(self.device, val, self.val_groups, labeler,
                                                    output_folder=c["output_folder"],
                                                    scale_shift=getattr(self, "scale_shift", None))
            if c["train_or_eval"] == "eval":
                return trainer.evaluate(c["test_loss_fxn"], self.device, val, labeler,
                                        output_folder=c["output_folder"], samples=self.val_samples,
                                        scale_shift=getattr(self, "scale_shift", None),
                                        dump_embeddings=c.get("dump_embeddings", False),
                                        compute_total_energy=c.get("compute_total_energy", False),
                                        basis_name=c.get("pyscf_basis"), xc=c.get("functional", "b3lyp"),
                                        hf_basis_file=c.get("hf_basis_file"))
            if c["distribute_graphs"] and getattr(self, "partition_sample", None) is None:
                # molecule batches split over ranks: one block-sparse shard folder per batch
                from ..parallel.infer import write_partition_hamiltonian

                paths = []
                with torch.no_grad():
                    for i, b in enumerate(val):
                        no, eo = head(backbone(b), b)
                        paths.append(write_partition_hamiltonian(os.path.join(c["output_folder"], f"batch_{i:04d}"),
                                                                 b, no[0], eo[0], labeler))
                return paths
            if c["distribute_graphs"]:
                b = val[0]
                s = self.partition_sample
                e = b.global_edge_ids.cpu().numpy()
                with torch.no_grad():
                    no, eo = head(backbone(b), b)
                from ..parallel.infer import write_partition_hamiltonian

                return write_partition_hamiltonian(c["output_folder"], b, no[0], eo[0], labeler,
                                                   global_src=s.src[e], global_dst=s.dst[e])
            if len(val) == 1:
                return trainer.infer(self.device, val[0].to(self.device), labeler, output_folder=c["output_folder"])
            # every batch of the evaluation set (reference ``splittrainer.py:825-1148``), one
            # block-sparse shard folder per batch
            return [trainer.infer(self.device, bt.to(self.device), labeler,
                                  output_folder=os.path.join(c["output_folder"], f"batch_{i:04d}"))
                    for i, bt in enumerate(val)]
        except BaseException:
            # the other ranks may be inside a collective this rank will never join: leave
            # without the closing barrier (their process-group timeout ends their wait)
            self.close(sync=False)
            raise
        finally:
            self.close()

    def close(self, sync=True):
        pdist.cleanup_process_group(sync_barrier=sync and self.world_size > 1)
