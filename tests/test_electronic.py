"""Orbital energies / densities from Fock matrices, and the workflow's eval output."""
import numpy as np
import scipy.linalg

from maloq_b200.eval import electronic


def _system(n=12, seed=0):
    rng = np.random.default_rng(seed)
    A = rng.standard_normal((n, n))
    F = 0.5 * (A + A.T)
    B = rng.standard_normal((n, n)) * 0.2
    S = np.eye(n) + 0.5 * (B + B.T)
    S = S @ S.T / np.linalg.norm(S, 2) + 0.2 * np.eye(n)
    return F, S


def test_generalised_orbitals_match_scipy_and_density_is_idempotent():
    F, S = _system()
    e, C = electronic.orbitals(F, S, tol=1e-8)
    assert np.allclose(e, scipy.linalg.eigh(F, S, eigvals_only=True), atol=1e-9)
    assert np.allclose(C.T @ S @ C, np.eye(len(e)), atol=1e-9)
    P = electronic.closed_shell_density(C, 8)
    assert np.allclose(P @ S @ P, 2.0 * P, atol=1e-9)
    out = electronic.summary(F, S, 8, tol=1e-8)
    assert abs(out["band_energy"] - 2 * e[:4].sum()) < 1e-12 and abs(out["gap"] - (e[4] - e[3])) < 1e-12


def test_near_dependent_overlap_directions_are_dropped():
    F, S = _system(10, seed=1)
    v = np.linalg.eigh(S)[1][:, 0]
    S2 = S - (v @ S @ v - 1e-4) * np.outer(v, v)  # one overlap eigenvalue -> 1e-4
    e, C = electronic.orbitals(F, S2, tol=1e-1)
    assert len(e) < 10 and np.allclose(C.T @ S2 @ C, np.eye(len(e)), atol=1e-8)


def test_workflow_eval_writes_orbital_metrics(tmp_path):
    from maloq.train_utils import training_workflow

    cfg = dict(dataset_name="synthetic_small", num_structures=6, batch_size=3, num_epochs=1, l_embedding_dim=8,
               num_mp_layers=1, num_distance_basis=8, rcut_orbitals=2.5, rcut_gaussian=5.0, mmax=2,
               output_folder=str(tmp_path), device="cpu", log_every=0)
    training_workflow.TrainingWorkflow(cfg).run()
    training_workflow.TrainingWorkflow(dict(cfg, train_or_eval="eval", restart_backbone=True,
                                            restart_head=True)).run()
    lines = (tmp_path / "model_fock_eval_0.txt").read_text().splitlines()
    assert lines[0].split("\t") == ["Index", "Total_MAE", "Eigenvalue_MAE", "Gap_Error", "Band_Energy_Error",
                                    "Num_Atoms"]
    vals = [float(x) for x in lines[1].split("\t")]
    assert np.isfinite(vals[1]) and np.isfinite(vals[2])


def test_embedding_dumps_projection_and_clusters(tmp_path):
    from maloq.train_utils import training_workflow
    from maloq_b200.analysis import embeddings

    cfg = dict(dataset_name="synthetic_small", num_structures=16, batch_size=4, num_epochs=1, l_embedding_dim=8,
               num_mp_layers=1, num_distance_basis=8, rcut_orbitals=2.5, rcut_gaussian=5.0, mmax=2,
               output_folder=str(tmp_path), device="cpu", log_every=0)
    training_workflow.TrainingWorkflow(cfg).run()
    training_workflow.TrainingWorkflow(dict(cfg, train_or_eval="eval", restart_backbone=True, restart_head=True,
                                            dump_embeddings=True)).run()
    folder = tmp_path / "embeddings"
    x, z = embeddings.load(folder)
    assert x.ndim == 3 and x.shape[1] == 25 and len(z) == len(x)
    f = embeddings.invariant_features(x)
    assert f.shape == (len(x), 5 * x.shape[2])
    out = embeddings.main([str(folder), "--method", "pca", "--clusters", "3"])
    rows = np.loadtxt(out, delimiter=",", skiprows=1)
    assert rows.shape == (len(x), 4) and set(np.unique(rows[:, 3])) <= {0, 1, 2}
    assert len(embeddings.project(f, "tsne")) == len(f)


def test_invariant_features_are_rotation_invariant():
    import torch

    from maloq_b200.analysis.embeddings import invariant_features
    from maloq_b200.core import sph

    rng = np.random.default_rng(0)
    x = rng.standard_normal((5, 25, 3))
    R = sph.euler_matrix(0.4, 1.1, -0.7)
    D = torch.block_diag(*[torch.tensor(sph.wigner_D_from_matrix(l, R)) for l in range(5)]).numpy()
    xr = np.einsum("ij,njc->nic", D, x)
    assert np.allclose(invariant_features(x), invariant_features(xr), atol=1e-10)


def test_eval_total_energy_column_without_pyscf(tmp_path):
    from maloq.train_utils import training_workflow

    cfg = dict(dataset_name="synthetic_small", num_structures=6, batch_size=3, num_epochs=1, l_embedding_dim=8,
               num_mp_layers=1, num_distance_basis=8, rcut_orbitals=2.5, rcut_gaussian=5.0, mmax=2,
               output_folder=str(tmp_path), device="cpu", log_every=0)
    training_workflow.TrainingWorkflow(cfg).run()
    rows = training_workflow.TrainingWorkflow(dict(cfg, train_or_eval="eval", restart_backbone=True, restart_head=True,
                                                   compute_total_energy=True)).run()
    header = (tmp_path / "model_fock_eval_0.txt").read_text().splitlines()[0].split("\t")
    assert "Total_Energy_Error" in header and len(rows[0]) == len(header)


def test_eval_hf_energy_column_with_own_integrals(tmp_path):
    """hf_basis_file: the evaluation adds the Hartree-Fock energy-functional error of the
    predicted Fock matrices, with this package's one-electron integrals (no PySCF)."""
    import numpy as np

    from maloq.train_utils import training_workflow

    def shell(kind, exps):
        return [f"{kind}   {len(exps)}   1.00"] + [f"  {e:.6f}   {1.0 / len(exps):.6f}" for e in exps]

    lines = []
    for sym, shells in (("H", ["S", "S", "P"]), ("C", ["S", "S", "S", "P", "P", "D"]), ("N", ["S", "S", "S", "P", "P", "D"]),
                        ("O", ["S", "S", "S", "P", "P", "D"])):
        lines.append(f"{sym}     0")
        for i, k in enumerate(shells):
            lines += shell(k, [6.0 / (i + 1), 1.2 / (i + 1)])
        lines.append("****")
    (tmp_path / "basis.g94").write_text("\n".join(lines) + "\n")
    cfg = dict(dataset_name="synthetic_small", num_structures=6, batch_size=3, num_epochs=1, l_embedding_dim=8,
               num_mp_layers=1, num_distance_basis=8, rcut_orbitals=2.5, rcut_gaussian=5.0, mmax=2,
               output_folder=str(tmp_path), device="cpu", log_every=0)
    training_workflow.TrainingWorkflow(cfg).run()
    rows = training_workflow.TrainingWorkflow(dict(cfg, train_or_eval="eval", restart_backbone=True, restart_head=True,
                                                   hf_basis_file=str(tmp_path / "basis.g94"))).run()
    header = (tmp_path / "model_fock_eval_0.txt").read_text().splitlines()[0].split("\t")
    assert header[-2] == "HF_Energy_Error" and len(rows[0]) == len(header)
    assert all(np.isfinite(r[-2]) and r[-2] >= 0 for r in rows)
