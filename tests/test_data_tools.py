"""Dataset tools (CPU): ORCA runs -> ASE database, linear energy references, scale/shift."""
import numpy as np
import torch

from maloq_b200.data import asedb, readers, tools
from maloq_b200.data.basis_sets import get_basis


def _orca_text(F, energy):
    from tests.test_cp2k_readers import _orca_block

    lines = ["junk", "---------------------------------", "CARTESIAN COORDINATES (ANGSTROEM)",
             "---------------------------------", "  H      0.000000    0.000000    0.740000",
             "  O      0.100000   -0.200000    0.000000", "", " BASIS SET INFORMATION",
             "Group   1 Type H   : 4s1p contracted to 2s1p pattern {31/1}",
             "Group   2 Type O   : 7s4p1d contracted to 3s2p1d pattern {511/31/1}", "",
             "TOTAL SCF ENERGY", "----------------", "",
             f"Total Energy       :        {energy:.11f} Eh           -2078.97 eV", "", "FOCK", ""]
    return "\n".join(lines + _orca_block(F) + ["", "end"]) + "\n"


def test_orca_runs_to_ase_database(tmp_path):
    rng = np.random.default_rng(0)
    Fs = []
    for k in range(3):
        F = np.round(rng.standard_normal((19, 19)), 6)
        F = F + F.T
        Fs.append(F)
        d = tmp_path / (f"run{k}_0_1" if k == 1 else f"run{k}")
        d.mkdir()
        (d / "orca.out").write_text(_orca_text(F, -76.0 - k))
    out = str(tmp_path / "mols.db")
    runs = [str(tmp_path / (f"run{k}_0_1" if k == 1 else f"run{k}")) for k in range(3)]
    assert tools.main(["orca-to-db", out] + runs) is None
    ds = asedb.ASEDataset(out)
    assert len(ds) == 3
    r = ds[1]
    assert list(r["atomic_numbers"]) == [1, 8] and r["folder_name"] == "run1_0_1"
    assert abs(r["energies"] + 77.0) < 1e-9
    ref = readers.reorder_orbitals(Fs[1], [1, 8], {1: [0, 0, 1], 8: [0, 0, 0, 1, 1, 2]}, "orca")
    assert np.allclose(r["fock_matrix"], ref, atol=1e-5)


def test_linear_references_recover_coefficients(tmp_path):
    rng = np.random.default_rng(1)
    coeff = {1: -0.5, 6: -37.8, 8: -75.0}
    basis = get_basis("def2_svp_nabla")
    mols = []
    for _ in range(20):
        z = rng.choice([1, 6, 8], size=int(rng.integers(3, 8))).astype(np.int32)
        E = sum(coeff[int(a)] for a in z) + rng.normal() * 1e-6
        n = sum(sum(2 * l + 1 for l in basis[int(a)]) for a in z)
        mols.append((z, rng.uniform(0, 6, (len(z), 3)), E, np.zeros((len(z), 3)), np.eye(n), np.eye(n), np.eye(n)))
    path = str(tmp_path / "nabla.db")
    readers.write_nabladft(path, mols)
    out = str(tmp_path / "lin.npz")
    tools.main(["lin-ref", path, out, "--dataset-name", "nablaDFT"])
    c = np.load(out)["coeff"]
    for z, v in coeff.items():
        assert abs(c[z] - v) < 1e-4, (z, c[z])


def test_scale_shift_table_matches_workflow_layout(tmp_path):
    from maloq_b200.data import datasets

    lab = datasets.labeler_for("small")
    samples, _ = datasets.build_dataset("small", 4, dict(sphere_channels=8, hidden_channels=8, lmax=4, mmax=2,
                                                          cutoff=5.0, num_layers=1, num_distance_basis=8,
                                                          edge_channels=8), labeler=lab)
    t = tools.scale_shift_table(samples, lab)
    assert set(t) == {"element_scalar_means", "element_scalar_stds", "scalar_irrep_indices"}
    z = int(samples[0].z[0])
    rows = torch.cat([s.node_y[0][torch.as_tensor(s.z == z)] for s in samples])
    idx = torch.tensor(t["scalar_irrep_indices"])
    assert torch.allclose(t["element_scalar_means"][z], rows[:, idx].float().mean(0), atol=1e-6)


def test_pooled_linear_references_and_statistics(tmp_path):
    """lin-ref over several ASE databases with random subsampling, then dataset statistics of
    the reference-subtracted energies and the forces."""
    import pickle

    rng = np.random.default_rng(2)
    coeff = {1: -0.5, 6: -37.8, 8: -75.0}
    paths, all_e, all_f = [], [], []
    for k in range(2):
        rows = []
        for _ in range(15):
            z = rng.choice([1, 6, 8], size=int(rng.integers(3, 8)))
            noise = rng.normal() * 1e-3
            f = rng.normal(size=(len(z), 3))
            rows.append({"numbers": z, "positions": rng.uniform(0, 5, (len(z), 3)), "forces": f,
                         "data": {"total_energy [Eh]": sum(coeff[int(a)] for a in z) + noise}})
            all_e.append(noise)
            all_f.append(f)
        p = str(tmp_path / f"part{k}.db")
        asedb.write_asedb(p, rows)
        paths.append(p)
    out = str(tmp_path / "lin.npz")
    tools.main(["lin-ref"] + paths + [out, "--dataset-name", "ase", "--subsample", "24", "--seed", "3"])
    c = np.load(out)["coeff"]
    for z, v in coeff.items():
        assert abs(c[z] - v) < 5e-3, (z, c[z])
    mols = tools.pooled_molecules(paths, "ase", subsample=24, seed=3)
    assert len(mols) == 24
    assert len({round(m[1], 12) for m in mols}) == 24  # drawn without replacement
    assert len(tools.pooled_molecules(paths, "ase", subsample=None)) == 30
    # statistics of one database with the exact references
    np.savez(str(tmp_path / "exact.npz"), coeff=np.array([0, -0.5, 0, 0, 0, 0, -37.8, 0, -75.0]))
    tools.main(["stats", paths[0], str(tmp_path / "st"), "--dataset-name", "ase", "--lin-ref",
                str(tmp_path / "exact.npz")])
    st = pickle.load(open(tmp_path / "st" / "stats.pkl", "rb"))
    e, f = np.array(all_e[:15]), np.concatenate(all_f[:15])
    assert abs(st["energy_mean"] - e.mean()) < 1e-9 and abs(st["energy_std"] - e.std()) < 1e-9
    assert abs(st["force_rms"] - np.sqrt(np.mean(f ** 2))) < 1e-12
    assert abs(st["force_md"] - np.linalg.norm(f, axis=1).mean()) < 1e-12
    h = np.load(tmp_path / "st" / "energy_histogram.npz")
    assert h["hist"].sum() == 15 and len(h["bins"]) == 101
    assert (tmp_path / "st" / "force_norm_histogram.npz").exists()


def test_open_shell_scale_shift_has_one_table_per_spin():
    from maloq_b200.data import datasets

    lab = datasets.labeler_for("small")
    samples, _ = datasets.build_dataset("small", 3, dict(sphere_channels=8, hidden_channels=8, lmax=4, mmax=2,
                                                          cutoff=5.0, num_layers=1, num_distance_basis=8,
                                                          edge_channels=8), labeler=lab)
    for s in samples:  # a second spin channel: alpha + 1
        s.node_y = torch.cat([s.node_y, s.node_y + 1.0])
    t = tools.scale_shift_table(samples, lab)
    assert {"element_scalar_means_alpha", "element_scalar_means_beta", "element_scalar_stds_alpha",
            "element_scalar_stds_beta", "scalar_irrep_indices"} == set(t)
    z = int(samples[0].z[0])
    assert torch.allclose(t["element_scalar_means_beta"][z], t["element_scalar_means_alpha"][z] + 1.0, atol=1e-5)
    assert torch.allclose(t["element_scalar_stds_beta"][z], t["element_scalar_stds_alpha"][z], atol=1e-5)


def test_workflow_scale_shift_shifts_each_spin_channel(tmp_path):
    """Open-shell targets keep both spin channels, each shifted by its own table; the saved
    file has the per-spin keys and is read back on the next run."""
    from maloq_b200.data import datasets
    from maloq_b200.train.workflow import TrainingWorkflow

    lab = datasets.labeler_for("small")
    kw = dict(sphere_channels=8, hidden_channels=8, lmax=4, mmax=2, cutoff=5.0, num_layers=1, num_distance_basis=8,
              edge_channels=8)
    samples, _ = datasets.build_dataset("small", 3, kw, labeler=lab)
    for s in samples:
        s.node_y = torch.cat([s.node_y, s.node_y + 1.0])
    orig = [s.node_y.clone() for s in samples]
    wf = TrainingWorkflow(dict(dataset_name="synthetic_small", output_folder=str(tmp_path), device="cpu",
                               scale_and_shift=True))
    wf._apply_scale_shift(samples, samples, lab, "osh")
    d = torch.load(tmp_path / "element_scale_shifts_osh.pt", weights_only=False)
    assert "element_scalar_means_beta" in d
    for s, o in zip(samples, orig):
        assert s.node_y.shape == o.shape
        # beta = alpha + 1 and beta's means = alpha's + 1: the shifted scalar entries agree
        assert torch.allclose(s.node_y[0][:, wf.scale_shift.scalar_idx], s.node_y[1][:, wf.scale_shift.scalar_idx],
                              atol=1e-5)
    again = [s.node_y.clone() for s in samples]
    for s, o in zip(samples, orig):
        s.node_y = o.clone()
    wf._apply_scale_shift(samples, samples, lab, "osh")  # loads the saved tables
    for s, a in zip(samples, again):
        assert torch.allclose(s.node_y, a, atol=1e-6)
