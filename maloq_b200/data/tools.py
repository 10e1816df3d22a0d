"""Dataset tools: database builders and target statistics, as standalone commands.

    python -m maloq_b200.data.tools orca-to-db OUT.db RUN_DIR [RUN_DIR ...] [--unrestricted]
    python -m maloq_b200.data.tools lin-ref DATASET [DATASET ...] OUT.npz [--dataset-name nablaDFT|QM7|ase]
                                            [--subsample N] [--seed S]
    python -m maloq_b200.data.tools stats DATASET OUT_DIR [--lin-ref LIN.npz] [--dataset-name ...]
    python -m maloq_b200.data.tools scale-shift DATASET OUT.pt [--dataset-name ...] [--num N]

* ``orca-to-db``: every directory holding an ORCA output (``*.out``) becomes one row of an ASE
  database (the format the OMol folders use): positions and atomic numbers, and in ``data``
  the Fock matrix converted to e3nn orbital order (``fock_matrix``; [2, n, n] for
  unrestricted runs), ``total_energy [Eh]``, ``is_open_shell``, ``charge``,
  ``spin_multiplicity`` and ``folder_name`` (reference
  ``dataset_utils/make_omol_database_raw.py``).  The basis shell order is the one ORCA prints.
* ``lin-ref``: per-element linear energy references - the least-squares fit of the total
  energies on the element counts, ``E ~ sum_Z n_Z(molecule) coeff[Z]`` - saved as
  ``coeff[Z]`` (the table the workflow subtracts from energy targets; reference
  ``dataset_utils/compute_lin_ref_nabla.py``).  Several databases (or folders of ASE databases)
  can be pooled; ``--subsample N`` draws N molecules at random, taking them from the databases in
  the order given until N are drawn (reference ``compute_lin_ref_omol_multi``).
* ``stats``: energy and force statistics of a dataset after the linear references are
  subtracted - energy mean and standard deviation, force RMS and mean force norm, mean atom count
  (``stats.pkl``), and 100-bin histograms of energies and force norms
  (``energy_histogram.npz``, ``force_norm_histogram.npz``; reference ``compute_stats``).
* ``scale-shift``: per-element means and standard deviations of the l = 0 on-site (node)
  label entries over a dataset, saved with the key names the workflow loads
  (``element_scalar_means``, ``element_scalar_stds``, ``scalar_irrep_indices``; reference
  ``dataset_utils/get_scale_shift.py``).
"""

from __future__ import annotations

import argparse
import glob
import os

import numpy as np
import torch


# ------------------------------------------------------------------ ORCA runs -> ASE database
def orca_runs_to_db(out_path, run_dirs, unrestricted=None, charge=None, spin_multiplicity=None):
    """One ASE-database row per ORCA run directory; returns the number of rows written.  Charge
    and multiplicity default to the ``..._<charge>_<multiplicity>`` suffix of the run's folder
    (or a parent's; 0 and 1 without one), and a multiplicity above 1 means an unrestricted run
    (two Fock matrices) unless ``unrestricted`` says otherwise."""
    from .asedb import write_asedb
    from .readers import charge_and_multiplicity_from_path, read_orca_output, reorder_orbitals

    rows = []
    for d in run_dirs:
        outs = sorted(glob.glob(os.path.join(d, "*.out")))
        if not outs:
            continue
        q_path, m_path = charge_and_multiplicity_from_path(outs[0])
        q = q_path if charge is None else charge
        mult = m_path if spin_multiplicity is None else spin_multiplicity
        uhf = (mult > 1) if unrestricted is None else bool(unrestricted)
        r = read_orca_output(outs[0], unrestricted=uhf)
        z = np.asarray(r["z"], dtype=np.int64)
        basis = r["basis"]
        if uhf:
            fock = np.stack([reorder_orbitals(r["fock"][k], z, basis, "orca") for k in ("alpha", "beta")])
        else:
            fock = reorder_orbitals(r["fock"], z, basis, "orca")
        data = {"fock_matrix": fock.astype(np.float32),
                "total_energy [Eh]": r["energy"] if r["energy"] is not None else 0.0,
                "is_open_shell": uhf, "charge": int(q), "spin_multiplicity": int(mult),
                "folder_name": os.path.basename(os.path.normpath(d))}
        if r["orbital_energies"]:
            data["orbital_energies [Eh]"] = np.stack(r["orbital_energies"]) if len(
                {len(e) for e in r["orbital_energies"]}) == 1 else r["orbital_energies"][0]
        rows.append({"numbers": z, "positions": np.asarray(r["pos"]), "energy": r["energy"], "data": data})
    if rows:
        write_asedb(out_path, rows)
    return len(rows)


# ------------------------------------------------------------------ statistics
def linear_energy_references(numbers_list, energies):
    """coeff[Z] minimising ||E - counts @ coeff||^2 over molecules (least squares)."""
    zmax = max(int(np.max(z)) for z in numbers_list)
    A = np.stack([np.bincount(np.asarray(z, dtype=np.int64), minlength=zmax + 1) for z in numbers_list])
    return np.linalg.lstsq(A.astype(np.float64), np.asarray(energies, dtype=np.float64), rcond=None)[0]


def scale_shift_table(samples, labeler):
    """Per-element means / stds of the l = 0 node label entries of ``samples`` (targets in
    ``node_y`` [spins, N, D]), in the workflow's file layout.  Open-shell targets (two spin
    channels) give one table per channel, keys suffixed ``_alpha`` / ``_beta`` (reference
    ``get_scale_shift.py:256-268``)."""
    from .targets import ScaleShift

    ss = ScaleShift(labeler, samples)
    idx = ss.scalar_idx
    spins = int(samples[0].node_y.shape[0]) if samples else 1
    out = {"scalar_irrep_indices": idx.tolist()}
    for k in range(spins):
        means, stds = {}, {}
        for z in ss.means:
            rows = torch.cat([s.node_y[k][torch.as_tensor(s.z == z)][:, idx] for s in samples]).float()
            means[z] = rows.mean(0)
            stds[z] = rows.std(0, unbiased=False)
        suffix = "" if spins == 1 else ("_alpha", "_beta")[k]
        out["element_scalar_means" + suffix] = means if spins > 1 else ss.means
        out["element_scalar_stds" + suffix] = stds
    return out


def _load(path, name, num=None):
    from . import readers

    cfg = {"rcut_orbitals": 3.0, "num_structures": num}
    if name == "nablaDFT":
        return readers.load_nabladft(path, {k: v for k, v in cfg.items() if v is not None})
    if name == "QM7":
        return readers.load_qm7(path, cfg)
    return readers.load_ase_entries([{"db_file": path, "start_idx": 0, "end_idx": num}], cfg)


def _db_files(path):
    if os.path.isdir(path):
        return sorted(glob.glob(os.path.join(path, "*.db")))
    return [path]


def _molecules(path, name, num=None):
    """(atomic numbers, total energy, forces or None) of the first ``num`` molecules of one
    dataset (a nablaDFT database, a QM7 / ASE database, or a folder of ASE databases)."""
    if name == "nablaDFT":
        from .readers import NablaDFTDatabase

        db = NablaDFTDatabase(path)
        n = len(db) if num is None else min(num, len(db))
        rows = [db[i] for i in range(n)]
        return [(np.asarray(r[0]), float(np.asarray(r[2]).reshape(-1)[0]), np.asarray(r[3], dtype=np.float64))
                for r in rows]
    from .asedb import AseDb

    out = []
    for f in _db_files(path):
        left = None if num is None else num - len(out)
        if left is not None and left <= 0:
            break
        db = AseDb(f)
        for r in db.rows(0, left):
            d = r["data"]
            if name == "QM7":
                e = float(np.asarray(d.get("energy", r["energy"])).reshape(-1)[0])
                fr = d.get("forces", r["forces"])
            else:
                e = float(d.get("total_energy [Eh]", r["energy"]))
                fr = r["forces"]
            out.append((r["numbers"], e, None if fr is None else np.asarray(fr, dtype=np.float64).reshape(-1, 3)))
        db.close()
    return out


def _energies(path, name, num=None):
    mols = _molecules(path, name, num)
    return [m[0] for m in mols], [m[1] for m in mols]


def pooled_molecules(paths, name, subsample=None, seed=0):
    """Molecules of several datasets; with ``subsample``, N drawn at random without replacement,
    from the datasets in the given order until N are drawn."""
    rng = np.random.default_rng(seed)
    out = []
    for p in paths:
        mols = _molecules(p, name)
        if subsample is not None:
            left = subsample - len(out)
            if left <= 0:
                break
            if len(mols) > left:
                mols = [mols[i] for i in sorted(rng.choice(len(mols), size=left, replace=False))]
        out += mols
    return out


def dataset_statistics(mols, coeff=None, bins=100):
    """Energy / force statistics after subtracting the linear references ``coeff[Z]``."""
    e = np.array([m[1] - (float(np.sum(np.asarray(coeff)[np.asarray(m[0])])) if coeff is not None else 0.0)
                  for m in mols])
    f = [m[2] for m in mols if m[2] is not None]
    f = np.concatenate(f) if f else np.zeros((0, 3))
    fn = np.linalg.norm(f, axis=-1)
    st = {"energy_mean": float(e.mean()), "energy_std": float(e.std()),
          "force_rms": float(np.sqrt(np.mean(f ** 2))) if len(f) else float("nan"),
          "force_md": float(fn.mean()) if len(fn) else float("nan"),
          "avg_num_atoms": float(np.mean([len(m[0]) for m in mols]))}
    hists = {"energy": np.histogram(e, bins=bins), "force_norm": np.histogram(fn, bins=bins) if len(fn) else None}
    return st, hists


def write_statistics(out_dir, st, hists):
    import pickle

    os.makedirs(out_dir, exist_ok=True)
    with open(os.path.join(out_dir, "stats.pkl"), "wb") as fh:
        pickle.dump(st, fh)
    for key, fname in (("energy", "energy_histogram.npz"), ("force_norm", "force_norm_histogram.npz")):
        if hists[key] is not None:
            np.savez(os.path.join(out_dir, fname), hist=hists[key][0], bins=hists[key][1])


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    a = sub.add_parser("orca-to-db")
    a.add_argument("out")
    a.add_argument("runs", nargs="+")
    a.add_argument("--unrestricted", action="store_true", default=None)
    a.add_argument("--charge", type=int, default=None)
    a.add_argument("--multiplicity", type=int, default=None)
    b = sub.add_parser("lin-ref")
    b.add_argument("datasets", nargs="+")
    b.add_argument("out")
    b.add_argument("--dataset-name", default="nablaDFT")
    b.add_argument("--num", type=int, default=None)
    b.add_argument("--subsample", type=int, default=None)
    b.add_argument("--seed", type=int, default=0)
    st = sub.add_parser("stats")
    st.add_argument("dataset")
    st.add_argument("out_dir")
    st.add_argument("--dataset-name", default="nablaDFT")
    st.add_argument("--lin-ref", default=None)
    st.add_argument("--num", type=int, default=None)
    c = sub.add_parser("scale-shift")
    c.add_argument("dataset")
    c.add_argument("out")
    c.add_argument("--dataset-name", default="nablaDFT")
    c.add_argument("--num", type=int, default=None)
    args = ap.parse_args(argv)
    if args.cmd == "orca-to-db":
        n = orca_runs_to_db(args.out, args.runs, args.unrestricted, args.charge, args.multiplicity)
        print(f"wrote {n} rows to {args.out}")
    elif args.cmd == "lin-ref":
        if args.subsample is None and len(args.datasets) == 1:
            mols = _molecules(args.datasets[0], args.dataset_name, args.num)
        else:
            mols = pooled_molecules(args.datasets, args.dataset_name, args.subsample, args.seed)
        coeff = linear_energy_references([m[0] for m in mols], [m[1] for m in mols])
        np.savez(args.out, coeff=coeff)
        print(f"linear references for {len(mols)} molecules -> {args.out}")
    elif args.cmd == "stats":
        mols = _molecules(args.dataset, args.dataset_name, args.num)
        coeff = np.load(args.lin_ref)["coeff"] if args.lin_ref else None
        st, hists = dataset_statistics(mols, coeff)
        write_statistics(args.out_dir, st, hists)
        print(", ".join(f"{k}: {v:.6g}" for k, v in st.items()))
    else:
        samples, lab = _load(args.dataset, args.dataset_name, args.num)
        torch.save(scale_shift_table(samples, lab), args.out)
        print(f"scale/shift of {len(samples)} molecules -> {args.out}")


if __name__ == "__main__":
    main()
