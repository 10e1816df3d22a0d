"""Train / evaluate / infer loops (reference ``train_utils/splittrainer.py``).

:class:`SplitTrainer` keeps the reference's constructor and method names.  What differs:

* the step is device-timed with CUDA events (no host ``perf_counter`` around async work);
* data-parallel gradients go through :class:`maloq_b200.parallel.dp.GradSync`, which
  reduces bucket by bucket while backward still runs (the reference all-reduces every
  parameter after backward, ``splittrainer.py:204-218``);
* the Fock loss is one fused masked kernel that also writes its gradient;
* batches are prefetched to the device on a side stream from pinned host memory;
* checkpoints carry the epoch, scheduler and RNG state in addition to the reference's
  ``{backbone|head}.pt`` files, so resume continues where it stopped.
"""

from __future__ import annotations

import os
import time

import numpy as np
import torch
import torch.distributed as dist

from ..ops import loss as loss_ops
from . import checkpoint as ckpt


def _rank():
    return dist.get_rank() if dist.is_available() and dist.is_initialized() else 0


def _world():
    return dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1


class Prefetcher:
    """Copies host batches to the device on a side stream, one batch ahead."""

    def __init__(self, batches, device):
        self.batches, self.device = batches, torch.device(device)
        self.stream = torch.cuda.Stream(device=self.device) if self.device.type == "cuda" else None

    def __iter__(self):
        if self.stream is None:
            for b in self.batches:
                yield b.to(self.device)
            return
        it = iter(self.batches)
        nxt = None
        try:
            nxt = self._issue(next(it))
        except StopIteration:
            return
        for b in it:
            cur, ev = nxt
            torch.cuda.current_stream(self.device).wait_event(ev)
            nxt = self._issue(b)
            yield cur
        cur, ev = nxt
        torch.cuda.current_stream(self.device).wait_event(ev)
        yield cur

    def _issue(self, b):
        with torch.cuda.stream(self.stream):
            d = b.to(self.device, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self.stream)
        return d, ev


class SplitTrainer:
    def __init__(self, backbone, head, head_irreps, save_frequency=10, run_id=None, run_name="noname",
                 mask_table=None, grad_sync=None, nan_guard=False, status_every=0, uncoupled_loss_transform=None):
        self.backbone, self.head, self.head_irreps = backbone, head, head_irreps
        self.save_frequency, self.run_name = save_frequency, run_name
        self.mask_table = mask_table
        self.grad_sync = grad_sync
        self.nan_guard = nan_guard
        # every ``status_every`` steps (0: only at the end of each epoch) the device error word
        # is read and a recorded timeout / bounds error raised on the host (CommTimeoutError,
        # BoundsError); reading it synchronises the device
        self.status_every = int(status_every)
        # compute_uncoupled_loss: outputs and targets go through get_H (matrix-element basis)
        # before the loss; the padding masks are the same in both bases (each CG block keeps
        # its index range)
        self.uncoupled = uncoupled_loss_transform
        self._steps = 0
        self.open_shell = getattr(head, "num_spins", 1) > 1
        self.history = {"train_node": [], "train_edge": [], "val_node": [], "val_edge": []}
        self.start_epoch = 0

    @staticmethod
    def check_status(where=""):
        """Raise the device error recorded by a kernel, if any (CUDA runs only)."""
        if torch.cuda.is_available() and torch.cuda.is_initialized():
            from ..ops import kernels

            kernels.check_device_status(where)

    # ------------------------------------------------------------------ one step
    def masks(self, batch):
        dev = batch.node_pair_type.device
        if getattr(self, "_mask_dev", None) is None or self._mask_dev.device != dev:
            self._mask_dev = self.mask_table.to(dev)  # copied to the device once, not every step
        return self._mask_dev, batch.node_pair_type, batch.edge_pair_type

    def forward_loss(self, batch, loss_fxn):
        emb = self.backbone(batch)
        out = self.head(emb, batch)
        if isinstance(out, dict):  # energy / force heads: one loss on the predicted quantity
            key, target = ("energies", batch.energy) if "energies" in out else ("forces", batch.forces)
            if target is None:
                raise ValueError(f"the batch carries no {key} targets")
            loss = loss_fxn(out[key], target.to(out[key].dtype))
            return loss, torch.zeros_like(loss), loss
        node_out, edge_out = out
        mt, npt, ept = self.masks(batch)
        spins = node_out.shape[0]
        lns, les, lts = [], [], []
        for s in range(spins):
            if spins == 1:  # a view whose backward allocates nothing (indexing [0] would)
                no, eo, nt, et = node_out.squeeze(0), edge_out.squeeze(0), batch.node_y[0], batch.y[0]
            else:
                no, eo, nt, et = node_out[s], edge_out[s], batch.node_y[s], batch.y[s]
            if self.uncoupled is not None:
                T = self.uncoupled
                no, eo = T.get_H(no), T.get_H(eo)
                with torch.no_grad():
                    nt, et = T.get_H(nt.to(no.dtype)), T.get_H(et.to(eo.dtype))
            ln, le, lt = loss_ops.fock_loss(no, eo, nt, et, mt, npt, ept, loss_fxn)
            lns.append(ln)
            les.append(le)
            lts.append(lt)
        return sum(lns) / spins, sum(les) / spins, sum(lts) / spins

    def train_step(self, batch, loss_fxn, optimizer, scheduler=None):
        ln, le, loss = self.forward_loss(batch, loss_fxn)
        if self.nan_guard and not torch.isfinite(loss).item():
            raise FloatingPointError(f"non-finite loss {loss.item()} - step skipped (inputs or parameters corrupted)")
        if self.grad_sync is not None:
            self.grad_sync.begin_step()
        loss.backward()
        if self.grad_sync is not None:
            self.grad_sync.finish()
        optimizer.step()
        optimizer.zero_grad(set_to_none=True)
        self._steps += 1
        if self.status_every and self._steps % self.status_every == 0:
            self.check_status(f"train step {self._steps}")
        if scheduler is not None and not hasattr(scheduler, "patience"):
            scheduler.step()
        return ln.detach(), le.detach(), loss.detach()

    # ------------------------------------------------------------------ loops
    def train(self, num_epochs, loss_fxn, optimizer, scheduler, device, train_loader, loss_target_string="fock_matrix",
              node_target_name="node_y", val_loader=None, edge_target_name="y", output_folder="outputs",
              step_every_epoch=False, min_lr=1e-10, log_every=1, **unused):
        rank = _rank()
        val_loader = val_loader or train_loader
        self.check_batch_consistency(len(train_loader), len(val_loader), device)
        os.makedirs(output_folder, exist_ok=True)
        for epoch in range(self.start_epoch, num_epochs):
            self.backbone.train()
            self.head.train()
            t0 = time.perf_counter()
            sn = torch.zeros((), device=device)
            se = torch.zeros((), device=device)
            for bi, batch in enumerate(Prefetcher(train_loader, device)):
                ln, le, loss = self.train_step(batch, loss_fxn, optimizer, scheduler)
                sn += ln
                se += le
                if rank == 0 and log_every and bi % log_every == 0:
                    print(f"--> Rank {rank} epoch {epoch + 1} batch {bi} loss: {loss.item():.6g}", flush=True)
            nb = max(1, len(train_loader))
            self.check_status(f"epoch {epoch + 1}")
            self.history["train_node"].append(sn.item() / nb)
            self.history["train_edge"].append(se.item() / nb)
            vn, ve, vt = self.validate(val_loader, loss_fxn, device)
            self.history["val_node"].append(vn)
            self.history["val_edge"].append(ve)
            if hasattr(scheduler, "patience"):
                scheduler.step(vt)
            elif step_every_epoch and scheduler is not None:
                scheduler.step()
            lr = optimizer.param_groups[0]["lr"]
            if rank == 0:
                print(f"Epoch {epoch + 1}, Train Loss: [node] {self.history['train_node'][-1]:.6g} "
                      f"[edge] {self.history['train_edge'][-1]:.6g}  Val: [node] {vn:.6g} [edge] {ve:.6g}  "
                      f"lr {lr:.3g}  time {time.perf_counter() - t0:.2f}s", flush=True)
            done = lr <= min_lr
            periodic = self.save_frequency and (epoch + 1) % self.save_frequency == 0  # 0: only at the end
            if rank == 0 and (periodic or done or epoch + 1 == num_epochs):
                self.save_training_state(epoch, optimizer, scheduler, output_folder)
            if done:
                print("Reached minimum learning rate, finished training.", flush=True)
                return
        return self.history

    @torch.no_grad()
    def validate(self, loader, loss_fxn, device):
        self.backbone.eval()
        self.head.eval()
        tot = torch.zeros(3, device=device, dtype=torch.float64)
        for batch in Prefetcher(loader, device):
            ln, le, lt = self.forward_loss(batch, loss_fxn)
            tot += torch.stack([ln, le, lt]).double()
        tot /= max(1, len(loader))
        if _world() > 1:
            dist.all_reduce(tot)
            tot /= _world()
        return tuple(tot.tolist())

    def check_batch_consistency(self, num_train_batches, num_val_batches, device):
        """All ranks must see the same number of batches (``splittrainer.py:1152-1170``)."""
        if _world() == 1:
            return
        t = torch.tensor([num_train_batches, num_val_batches], device=device if dist.get_backend() == "nccl" else "cpu")
        lst = [torch.zeros_like(t) for _ in range(_world())]
        dist.all_gather(lst, t)
        if not all(torch.equal(lst[0], x) for x in lst):
            raise ValueError(f"Mismatch in number of batches across ranks: {[x.tolist() for x in lst]}")

    def save_training_state(self, epoch, optimizer, scheduler, output_folder):
        ckpt.save_training_state(output_folder, self.backbone, self.head, optimizer, scheduler, epoch, self.history)

    # ------------------------------------------------------------------ eval / infer
    @torch.no_grad()
    def evaluate(self, loss_fxn, device, loader, labeler, output_folder="outputs", samples=None, scale_shift=None,
                 dump_embeddings=False, compute_total_energy=False, basis_name=None, xc="b3lyp",
                 hf_basis_file=None, **unused):
        """Per structure: Hamiltonian MAE, orbital-energy MAE (generalised with the overlap
        when the sample carries one, canonical orthogonalisation), HOMO-LUMO gap and band
        energy errors (closed shell, all-electron count), written to
        ``model_fock_eval_{rank}.txt`` (reference ``splittrainer.py:378-822``).

        ``hf_basis_file`` (a Gaussian94 basis file whose shells match the labels' basis) adds
        ``HF_Energy_Error``: the difference of the Hartree-Fock energy functionals
        E = 1/2 Tr[P (H + F)] + E_nn of the predicted and target Fock matrices, with this
        package's own one-electron integrals (no PySCF; for Kohn-Sham targets the XC correction
        is not included)."""
        from ..data.batch import collate

        hf_basis = None
        if hf_basis_file:
            from ..eval.integrals import parse_gaussian94

            with open(hf_basis_file) as fh:
                hf_basis = parse_gaussian94(fh.read())
            for zz, ls in labeler.orbital_basis.items():
                got = [l for l, *_ in hf_basis.get(zz, [])]
                if got != [l % 10 for l in ls]:
                    raise ValueError(f"hf_basis_file: element {zz} has shells {got}, the labels' basis {ls}")

        mol_of = None
        if compute_total_energy:
            try:
                from pyscf import gto

                def mol_of(s):
                    return gto.M(atom=[(int(z), tuple(p)) for z, p in zip(s.z, s.pos)], basis=basis_name or "def2-svp",
                                 charge=int(getattr(s, "charge", 0)), unit="Angstrom")
            except ImportError:
                print("compute_total_energy: PySCF is not installed; Total_Energy_Error is reported as nan",
                      flush=True)

        self.backbone.eval()
        self.head.eval()
        rank = _rank()
        rows = []
        for k, s in enumerate(samples):
            b = collate([s], labeler.table).to(device)
            emb = self.backbone(b)
            if dump_embeddings:
                from ..analysis.embeddings import dump

                dump(os.path.join(output_folder, "embeddings"), k, emb, b)
            out = self.head(emb, b)
            if isinstance(out, dict):  # energy / force heads
                if "energies" in out:
                    err = abs(float(out["energies"][0]) - float(b.energy[0])) if b.energy is not None else float("nan")
                    rows.append((k, err, float("nan"), s.num_nodes))
                else:
                    f = out["forces"].double().cpu().numpy()
                    err = float(np.abs(f - b.forces.double().cpu().numpy()).mean()) if b.forces is not None \
                        else float("nan")
                    rows.append((k, float("nan"), err, s.num_nodes))
                continue
            no, eo = out
            rows.append((k,) + self._fock_metrics(s, no[0], eo[0], b.node_y[0], b.y[0], labeler, scale_shift,
                                                   compute_total_energy, mol_of, xc, hf_basis))
        os.makedirs(output_folder, exist_ok=True)
        if rows and len(rows[0]) == 4:
            with open(os.path.join(output_folder, f"model_energy_eval_{rank}.txt"), "w") as f:
                f.write("Index\tEnergy_Error\tForce_MAE\tNum_Atoms\n")
                for r in rows:
                    f.write("\t".join(str(x) for x in r) + "\n")
            return rows
        with open(os.path.join(output_folder, f"model_fock_eval_{rank}.txt"), "w") as f:
            f.write("Index\tTotal_MAE\tEigenvalue_MAE\tGap_Error\tBand_Energy_Error\t"
                    + ("Total_Energy_Error\t" if compute_total_energy else "")
                    + ("HF_Energy_Error\t" if hf_basis is not None else "") + "Num_Atoms\n")
            for r in rows:
                f.write("\t".join(str(x) for x in r) + "\n")
        return rows

    @staticmethod
    def _fock_metrics(s, no, eo, ty, y, labeler, scale_shift, compute_total_energy, mol_of, xc, hf_basis=None):
        """Errors of one structure's predicted labels (no, eo) against its targets (ty, y):
        Hamiltonian MAE, orbital-energy MAE, gap and band-energy errors (and total energy)."""
        from ..eval import electronic

        if scale_shift is not None:
            no = scale_shift.unshift(no, s.z)
            ty = scale_shift.unshift(ty, s.z)
        bp = labeler.blocks_from_labels(s, no, eo)
        bt = labeler.blocks_from_labels(s, ty, y)
        Hp, Ht = bp.to_dense(), bt.to_dense()
        Hp = 0.5 * (Hp + Hp.T)
        S = getattr(s, "overlap", None)
        ne = electronic.n_electrons(s.z, getattr(s, "charge", 0))
        sp_, st_ = electronic.summary(Hp, S, ne), electronic.summary(Ht, S, ne)
        ep, et = sp_["eigenvalues"], st_["eigenvalues"]

        def err(key):
            return float("nan") if sp_[key] is None else abs(sp_[key] - st_[key])

        row = [float(np.abs(Hp - Ht).mean()), float(np.abs(ep - et).mean()), err("gap"), err("band_energy")]
        if compute_total_energy:
            te = float("nan")
            if mol_of is not None:
                mol = mol_of(s)
                te = abs(electronic.total_energy(mol, Hp, S, xc) - electronic.total_energy(mol, Ht, S, xc))
            row.append(te)
        if hf_basis is not None:
            from ..eval.integrals import hf_energy

            ep_ = hf_energy(Hp, s.z, s.pos, hf_basis, n_electrons=ne)["total"]
            et_ = hf_energy(0.5 * (Ht + Ht.T), s.z, s.pos, hf_basis, n_electrons=ne)["total"]
            row.append(abs(ep_ - et_))
        return tuple(row + [s.num_nodes])

    @torch.no_grad()
    def evaluate_partitioned(self, device, batches, groups, labeler, output_folder="outputs", scale_shift=None,
                             **unused):
        """Evaluation of molecule supergraphs split over the ranks: every rank runs its domain of
        each supergraph; the owned node rows and local edge rows are gathered to rank 0 (uneven,
        as objects), put back in the supergraph's order and cut into molecules, whose metrics
        rank 0 writes to ``model_fock_eval_0.txt`` (reference ``splittrainer.py:1270-1404``).
        ``groups[i]`` are the molecules of ``batches[i]`` in the order they were merged."""
        self.backbone.eval()
        self.head.eval()
        rank, world = _rank(), _world()
        rows = []
        k = 0
        for b, group in zip(batches, groups):
            no, eo = self.head(self.backbone(b), b)
            mine = (b.global_node_ids.cpu(), no[0].float().cpu(), b.global_edge_ids.cpu(), eo[0].float().cpu())
            parts = [mine]
            if world > 1:
                parts = [None] * world
                dist.all_gather_object(parts, mine)
            if rank != 0:
                k += len(group)
                continue
            n_all = sum(len(m.z) for m in group)
            e_all = sum(len(m.src) for m in group)
            node = torch.zeros(n_all, no.shape[-1])
            edge = torch.zeros(e_all, eo.shape[-1])
            for ids, nv, eids, ev in parts:
                node[ids] = nv
                edge[eids] = ev
            n0 = e0 = 0
            for m in group:
                n1, e1 = n0 + len(m.z), e0 + len(m.src)
                rows.append((k,) + self._fock_metrics(m, node[n0:n1].to(device), edge[e0:e1].to(device),
                                                      torch.as_tensor(m.node_y[0]).to(device),
                                                      torch.as_tensor(m.y[0]).to(device), labeler, scale_shift,
                                                      False, None, None))
                n0, e0, k = n1, e1, k + 1
        if rank == 0:
            os.makedirs(output_folder, exist_ok=True)
            with open(os.path.join(output_folder, "model_fock_eval_0.txt"), "w") as f:
                f.write("Index\tTotal_MAE\tEigenvalue_MAE\tGap_Error\tBand_Energy_Error\tNum_Atoms\n")
                for r in rows:
                    f.write("\t".join(str(x) for x in r) + "\n")
        return rows

    @torch.no_grad()
    def infer(self, device, batch, labeler, output_folder="outputs", partition=None, **unused):
        """Forward + label -> block-sparse Hamiltonian; every rank writes its own blocks
        (``hamiltonian_rank{r}.npz``) instead of gathering to rank 0."""
        from ..parallel.infer import write_partition_hamiltonian

        self.backbone.eval()
        self.head.eval()
        emb = self.backbone(batch)
        no, eo = self.head(emb, batch)
        return write_partition_hamiltonian(output_folder, batch, no[0], eo[0], labeler, partition)
