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
